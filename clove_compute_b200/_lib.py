"""ctypes binding of libclove_b200.so (the C ABI of include/clove/capi.h)."""
from __future__ import annotations

import ctypes
import os
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_PKG, "libclove_b200.so")

CLOVE_OK = 0
CLOVE_ERR_INVALID_ARG = 1
CLOVE_ERR_UNSUPPORTED = 2
CLOVE_ERR_CUDA = 3
CLOVE_ERR_NCCL = 4
CLOVE_ERR_DEVICE = 5
CLOVE_ERR_TIMEOUT = 6
INT4_GROUP_SIZE = 128

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_I8 = ctypes.c_int8
_SZ = ctypes.c_size_t

# name -> (argtypes, restype); mirrors include/clove/capi.h.
SIGNATURES = {
    "clove_version": ([], ctypes.c_char_p),
    "clove_last_error_string": ([], ctypes.c_char_p),
    "clove_get_device_error": ([_P], _I),
    "clove_gemm_fp16": ([_P, _P, _P, _I, _I, _I, _F, _F, _P], _I),
    "clove_gemm_fp16_batched": ([_P, _P, _P, _I, _I, _I, _I, _F, _F, _P], _I),
    "clove_gemm_int8": ([_P, _P, _P, _I, _I, _I, _F, _I8, _F, _I8, _P], _I),
    "clove_gemm_int8_noalloc": ([_P, _P, _P, _I, _I, _I, _F, _I8, _F, _I8, _P], _I),
    "clove_gemm_int8_rowcol": ([_P, _P, _P, _I, _I, _I, _P, _P, _P], _I),
    "clove_gemm_int4": ([_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _P], _I),
    "clove_flash_attention": ([_P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _I, _I, _P], _I),
    "clove_debug_int8_acc": ([_P, _P, _P, _I, _I, _I, _I8, _I8, _P], _I),
    "clove_debug_int4_group_acc": ([_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _P], _I),
    "clove_quantize_int4": ([_P, _I, _I, _P, _P, _P, _P], _I),
    "clove_swiglu_fused": ([_P, _P, _P, _P, _I, _I, _I, _P], _I),
    "clove_debug_stream_read": ([_P, _SZ, _P, _P], _I),
    "clove_debug_exp2_poly": ([_P, _P, _I, _P], _I),
    "clove_debug_peer_wait_timeout": ([_P, ctypes.c_ulonglong, _P], _I),
    "clove_debug_stream_k_plan": ([_I, _I, _I, _I, _P], _I),
    "clove_set_dispatch_override": ([_I, _I, _I], _I),
    "clove_set_weight_prefetch": ([_I], _I),
    "clove_describe_dispatch": ([_I, _I, _I, _I, ctypes.c_char_p, _SZ], _I),
    "clove_nsplit_col_begin": ([_I, _I, _I], _I),
    "clove_nsplit_get_unique_id": ([_P], _I),
    "clove_nsplit_init": ([_P, _I, _I, _P], _I),
    "clove_nsplit_destroy": ([_P], _I),
    "clove_nsplit_rank": ([_P, _P, _P], _I),
    "clove_nsplit_register_output": ([_P, _P, _SZ], _I),
    "clove_nsplit_register_output_multicast": ([_P, _P, _P, _SZ], _I),
    "clove_nsplit_unregister_output": ([_P, _P], _I),
    "clove_nsplit_gemm_fp16": ([_P, _P, _P, _P, _P, _I, _I, _I, _F, _I, _P], _I),
    "clove_nsplit_gemm_int4": ([_P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P], _I),
    "clove_nsplit_gemm_int8_rowcol": ([_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P], _I),
}


class CloveError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"clove error {code}: {msg}")
        self.code = code


_lock = threading.Lock()
_lib = None


def library_path() -> str:
    return _LIB_PATH


def lib():
    """The loaded library. Raises if it was not built (``python -m clove_compute_b200.build``)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_LIB_PATH):
                raise ImportError(
                    f"{_LIB_PATH} is missing: build it with `python -m clove_compute_b200.build`")
            l = ctypes.CDLL(_LIB_PATH)
            for name, (args, res) in SIGNATURES.items():
                fn = getattr(l, name)
                fn.argtypes = args
                fn.restype = res
            _lib = l
    return _lib


def check(rc: int) -> None:
    if rc != CLOVE_OK:
        msg = lib().clove_last_error_string().decode(errors="replace")
        raise CloveError(rc, msg)
