"""clove_compute_b200 -- B200 (sm_100a) GEMM hot path of the clove runtime.

Python mirror of the reference's ``include/clove/kernels/gemm.cuh`` API
(``gemm_fp16``, ``gemm_int8``, ``gemm_int4``, ``gemm_fp16_batched``) over the
C ABI in ``include/clove/capi.h``. Same names, argument meaning and row-major
layouts; torch CUDA tensors supply device memory and the current stream.
Every call runs a kernel of ``libclove_b200.so`` (built in-tree for sm_100a);
there is no CPU or library fallback -- a missing library raises.
"""
from __future__ import annotations

from ._lib import (CloveError, lib, library_path, INT4_GROUP_SIZE,  # noqa: F401
                   CLOVE_OK, CLOVE_ERR_INVALID_ARG, CLOVE_ERR_UNSUPPORTED, CLOVE_ERR_CUDA,
                   CLOVE_ERR_NCCL, CLOVE_ERR_DEVICE, CLOVE_ERR_TIMEOUT)
from .api import (gemm_fp16, gemm_fp16_batched, gemm_int8, gemm_int8_rowcol, gemm_int4,  # noqa: F401
                  debug_int8_acc, debug_int4_group_acc, debug_stream_read, debug_stream_k_plan,
                  debug_peer_wait_timeout, debug_exp2_poly, quantize_int4, swiglu_fused,
                  flash_attention,
                  set_dispatch_override, set_weight_prefetch,
                  describe_dispatch, device_error, version)
from .nsplit import NSplit, col_begin  # noqa: F401

__all__ = [
    "gemm_fp16", "gemm_fp16_batched", "gemm_int8", "gemm_int8_rowcol", "gemm_int4",
    "debug_int8_acc", "debug_int4_group_acc", "debug_stream_read", "debug_stream_k_plan",
    "debug_peer_wait_timeout", "debug_exp2_poly", "quantize_int4",
    "swiglu_fused", "flash_attention",
    "set_dispatch_override",
    "set_weight_prefetch",
    "describe_dispatch",
    "device_error", "version", "NSplit", "col_begin", "CloveError", "lib", "library_path",
    "INT4_GROUP_SIZE",
]
