"""ctypes binding of ``libchia_attn.so`` (declared in ``include/chia_attn.h``).

The library is built in-tree by ``chia_proj_b200.build`` and loaded from
``chia_proj_b200/_lib/``. There is no fallback: if the library is missing or
fails to load, importing the operators raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libchia_attn.so")

ABI_VERSION = 4
WORKSPACE_BYTES = 256
NOALLOC_SCRATCH_BYTES = 256
NOALLOC_MAX_UNITS = 1 << 30

DTYPE_BF16, DTYPE_F16 = 0, 1
NORM_SOFTMAX, NORM_SIGMOID, NORM_RELU = 0, 1, 2
MOD_NONE, MOD_SOFTCAP, MOD_ALIBI, MOD_TEMP = 0, 1, 2, 3

STATUS = {
    0: "CHIA_OK",
    1: "CHIA_ERR_INVALID_ARGUMENT",
    2: "CHIA_ERR_UNSUPPORTED",
    3: "CHIA_ERR_MISALIGNED",
    4: "CHIA_ERR_LAUNCH",
    5: "CHIA_ERR_DEVICE_TIMEOUT",
    6: "CHIA_ERR_NO_DEVICE",
}

EXPORTED_SYMBOLS = (
    "chia_attn_fwd",
    "chia_attn_fwd_noalloc",
    "chia_attn_visible_pairs",
    "chia_attn_tile_plan",
    "chia_attn_status_string",
    "chia_attn_abi_version",
    "chia_attn_decode",
    "chia_attn_decode_workspace_bytes",
    "chia_attn_bwd",
    "chia_attn_bwd_workspace_bytes",
)


class AttnParams(ctypes.Structure):
    """Mirror of ``chia_attn_params_t`` (include/chia_attn.h)."""

    _fields_ = [
        ("abi_version", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("norm", ctypes.c_int32),
        ("mod", ctypes.c_int32),
        ("heads_kv", ctypes.c_int32),
        ("batch", ctypes.c_int64),
        ("heads", ctypes.c_int64),
        ("seqlen_q", ctypes.c_int64),
        ("seqlen_kv", ctypes.c_int64),
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("o", ctypes.c_void_p),
        ("q_stride", ctypes.c_int64 * 3),
        ("k_stride", ctypes.c_int64 * 3),
        ("v_stride", ctypes.c_int64 * 3),
        ("o_stride", ctypes.c_int64 * 3),
        ("scale", ctypes.c_float),
        ("softcap", ctypes.c_float),
        ("sig_bias", ctypes.c_float),
        ("out_scale", ctypes.c_float),
        ("head_param", ctypes.c_void_p),
        ("win_left", ctypes.c_int64),
        ("win_right", ctypes.c_int64),
        ("block", ctypes.c_int64),
        ("prefix", ctypes.c_int64),
        ("dilation", ctypes.c_int64),
        ("status", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p),
        ("seq_offsets", ctypes.c_void_p),
        ("num_seqs", ctypes.c_int64),
        ("lse", ctypes.c_void_p),
        ("wait_limit_ns", ctypes.c_uint64),
    ]


class AttnGrads(ctypes.Structure):
    """Mirror of ``chia_attn_grads_t`` (include/chia_attn.h)."""

    _fields_ = [
        ("dout", ctypes.c_void_p),
        ("dout_stride", ctypes.c_int64 * 3),
        ("dq", ctypes.c_void_p),
        ("dk", ctypes.c_void_p),
        ("dv", ctypes.c_void_p),
        ("dq_stride", ctypes.c_int64 * 3),
        ("dk_stride", ctypes.c_int64 * 3),
        ("dv_stride", ctypes.c_int64 * 3),
    ]


class ChiaError(RuntimeError):
    """A non-zero ``chia_status`` returned by the library."""

    def __init__(self, code: int, what: str = ""):
        self.code = code
        name = STATUS.get(code, f"status {code}")
        super().__init__(f"{name}{': ' + what if what else ''}")


_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load the native library (once). Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with "
                    "`python -m chia_proj_b200.build` (nvcc, sm_100a)")
            lib = ctypes.CDLL(LIB_PATH)
            lib.chia_attn_fwd.argtypes = [ctypes.POINTER(AttnParams), ctypes.c_void_p]
            lib.chia_attn_fwd.restype = ctypes.c_int
            lib.chia_attn_fwd_noalloc.argtypes = [ctypes.POINTER(AttnParams), ctypes.c_void_p]
            lib.chia_attn_fwd_noalloc.restype = ctypes.c_int
            lib.chia_attn_decode.argtypes = [ctypes.POINTER(AttnParams), ctypes.c_void_p,
                                             ctypes.c_int64, ctypes.c_void_p]
            lib.chia_attn_decode.restype = ctypes.c_int
            lib.chia_attn_decode_workspace_bytes.argtypes = [ctypes.POINTER(AttnParams)]
            lib.chia_attn_decode_workspace_bytes.restype = ctypes.c_int64
            lib.chia_attn_bwd.argtypes = [ctypes.POINTER(AttnParams), ctypes.POINTER(AttnGrads),
                                          ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
            lib.chia_attn_bwd.restype = ctypes.c_int
            lib.chia_attn_bwd_workspace_bytes.argtypes = [ctypes.POINTER(AttnParams)]
            lib.chia_attn_bwd_workspace_bytes.restype = ctypes.c_int64
            lib.chia_attn_visible_pairs.argtypes = [ctypes.POINTER(AttnParams)]
            lib.chia_attn_visible_pairs.restype = ctypes.c_int64
            lib.chia_attn_tile_plan.argtypes = [
                ctypes.POINTER(AttnParams), ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64),
                ctypes.POINTER(ctypes.c_uint64)]
            lib.chia_attn_tile_plan.restype = ctypes.c_int
            lib.chia_attn_status_string.argtypes = [ctypes.c_int]
            lib.chia_attn_status_string.restype = ctypes.c_char_p
            lib.chia_attn_abi_version.argtypes = []
            lib.chia_attn_abi_version.restype = ctypes.c_int
            if lib.chia_attn_abi_version() != ABI_VERSION:
                raise ImportError(f"{LIB_PATH}: ABI version mismatch")
            _lib = lib
    return _lib


def check(code: int, what: str = "") -> None:
    if code != 0:
        raise ChiaError(code, what)
