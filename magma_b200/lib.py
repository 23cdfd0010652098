"""ctypes binding of libmagma_cuda.so (the C ABI declared in include/magma_cuda.h).

Every entry point returns a status code with the values of Magma's
``SW_PJRT_Error_Code`` (Sources/CXLARuntime/include/PJRTSimpleWrapper.h:32-50);
a non-zero status raises :class:`MagmaError` carrying the thread-local message
from ``magma_get_last_error_message`` — the way Magma's Swift runtime turns
PJRT shim codes into thrown errors (Sources/XLARuntime/XLARuntime.swift).

There is no fallback: if the shared library is missing or cannot load, every
op raises.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libmagma_cuda.so"

# status codes (SW_PJRT_Error_Code values)
OK = 0
INVALID_ARGUMENT = 3
DEADLINE_EXCEEDED = 4
RESOURCE_EXHAUSTED = 8
FAILED_PRECONDITION = 9
OUT_OF_RANGE = 11
UNIMPLEMENTED = 12
INTERNAL = 13
UNAVAILABLE = 14

STATUS_NAMES = {0: "OK", 1: "CANCELLED", 2: "UNKNOWN", 3: "INVALID_ARGUMENT",
                4: "DEADLINE_EXCEEDED", 5: "NOT_FOUND", 8: "RESOURCE_EXHAUSTED",
                9: "FAILED_PRECONDITION", 11: "OUT_OF_RANGE", 12: "UNIMPLEMENTED",
                13: "INTERNAL", 14: "UNAVAILABLE"}

# dtypes (SW_PJRT_Buffer_Type values)
S32 = 3
S64 = 4
F32 = 10
BF16 = 12

# reductions of the collectives
REDUCE_SUM = 0
REDUCE_MAX = 1
REDUCE_MIN = 2
REDUCE_AVG = 3
COMM_ID_BYTES = 128

# GEMM epilogues
EPI_NONE = 0
EPI_BIAS = 1
EPI_BIAS_GELU = 2
EPI_BIAS_RESIDUAL = 3
EPI_DGELU = 4
EPI_ACCUMULATE = 5
EPI_BIAS_RELU = 6
EPI_DRELU = 7
EPI_ROWSTATS = 8


class MagmaError(RuntimeError):
    """A failed C-ABI call: ``status`` is the code, ``message`` the text."""

    def __init__(self, fn: str, status: int, message: str | None):
        self.fn = fn
        self.status = status
        self.message = message or ""
        super().__init__(f"{fn} failed with {STATUS_NAMES.get(status, status)}: {self.message}")


_vp = C.c_void_p
_i64 = C.c_int64
_i32 = C.c_int32
_f = C.c_float
_sz = C.c_size_t

# name -> (restype, argtypes). restype None means magma_status_t.
SIGNATURES = {
    "magma_get_last_error_message": (C.c_char_p, []),
    "magma_clear_last_error_message": ("void", []),
    "magma_abi_version": (C.c_int32, []),
    "magma_device_count": (None, [C.POINTER(C.c_int32)]),
    "magma_init": (None, [_i32]),
    "magma_stream_create": (None, [C.POINTER(_vp)]),
    "magma_stream_destroy": (None, [_vp]),
    "magma_stream_synchronize": (None, [_vp]),
    "magma_malloc": (None, [C.POINTER(_vp), _sz]),
    "magma_free": (None, [_vp]),
    "magma_memcpy_h2d": (None, [_vp, _vp, _sz, _vp]),
    "magma_memcpy_d2h": (None, [_vp, _vp, _sz, _vp]),
    "magma_memset": (None, [_vp, _i32, _sz, _vp]),
    "magma_device_error_check": (None, [_vp, C.POINTER(C.c_int32)]),
    "magma_layernorm_fwd": (None, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _f, _i32, _i32, _vp]),
    "magma_layernorm_bwd_workspace_size": (_sz, [_i64, _i64]),
    "magma_layernorm_bwd": (None, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i32, _i32,
                                   _i32, _i32, _i32, _vp, _sz, _vp]),
    "magma_layernorm_bwd_noalloc": (None, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64,
                                           _i32, _i32, _i32, _i32, _i32, _vp]),
    "magma_layernorm_bwd_residual_workspace_size": (_sz, [_i64, _i64]),
    "magma_layernorm_bwd_residual": (None, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                            _i64, _i64, _i32, _i32, _i32, _vp, _sz, _vp]),
    "magma_gemm_workspace_size": (_sz, [_i64, _i64, _i64, _i32]),
    "magma_gemm": (None, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _i32, _i32,
                          _i32, _i32, _vp, _vp, _vp, _vp, _sz, _vp]),
    "magma_attention_fwd": (None, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64,
                                   C.POINTER(_i64), C.POINTER(_i64), _f, _i32, _i32, _vp]),
    "magma_attention_bwd_workspace_size": (_sz, [_i64, _i64, _i64, _i64, _i32]),
    "magma_attention_bwd": (None, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64,
                                   _i64, C.POINTER(_i64), C.POINTER(_i64), _f, _i32, _i32, _vp,
                                   _sz, _vp]),
    "magma_adam_step": (None, [_vp, _vp, _vp, _vp, _vp, _i64, _f, _f, _f, _f, _f, _i64, _f, _vp]),
    "magma_adam_step_multi": (None, [C.POINTER(_vp), C.POINTER(_vp), C.POINTER(_vp),
                                     C.POINTER(_vp), C.POINTER(_i64), _i32, _f, _f, _f, _f, _f,
                                     _i64, _f, _vp]),
    "magma_grad_norm_workspace_size": (_i64, [_i64]),
    "magma_grad_norm": (None, [_vp, _i64, _f, _vp, _vp, _i64, _vp]),
    "magma_grad_sumsq": (None, [_vp, _i64, _f, _vp, _vp, _i64, _vp]),
    "magma_grad_norm_combine": (None, [_vp, _i64, _vp, _vp]),
    "magma_adam_step_clipped": (None, [_vp, _vp, _vp, _vp, _vp, _i64, _f, _f, _f, _f, _f, _i64,
                                       _f, _vp, _f, _vp]),
    "magma_lr_warmup_cosine": (None, [_f, _f, _i64, _i64, _i64, C.POINTER(_f)]),
    "magma_embedding_fwd": (None, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp]),
    "magma_embedding_bwd": (None, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp]),
    "magma_embedding_bwd_workspace_size": (_i64, [_i64, _i64]),
    "magma_embedding_bwd_deterministic": (None, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i32,
                                                 _vp, _i64, _vp]),
    "magma_cross_entropy_fwd_bwd": (None, [_vp, _vp, _vp, _i64, _i64, _i64, _f, _i32, _vp]),
    "magma_cross_entropy_fwd_bwd_rowstats": (None, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _f,
                                                    _i32, _vp]),
    "magma_reduce_sum": (None, [_vp, _vp, _i64, _f, _vp]),
    "magma_mse_fwd_bwd": (None, [_vp, _vp, _vp, _vp, _i64, _f, _vp]),
    "magma_gelu_fwd": (None, [_vp, _vp, _i64, _i32, _vp]),
    "magma_gelu_bwd": (None, [_vp, _vp, _vp, _i64, _i32, _vp]),
    "magma_relu_fwd": (None, [_vp, _vp, _i64, _i32, _vp]),
    "magma_relu_bwd": (None, [_vp, _vp, _vp, _i64, _i32, _vp]),
    "magma_bias_grad_workspace_size": (_sz, [_i64, _i64]),
    "magma_bias_grad": (None, [_vp, _vp, _i64, _i64, _i64, _i32, _i32, _vp, _sz, _vp]),
    "magma_convert": (None, [_vp, _vp, _i64, _i32, _i32, _vp]),
    "magma_comm_unique_id": (None, [C.c_char_p, _sz]),
    "magma_comm_init_rank": (None, [C.POINTER(_vp), _i32, _i32, C.c_char_p, _i64]),
    "magma_comm_init_all": (None, [_i32, C.POINTER(_i32), C.POINTER(_vp)]),
    "magma_comm_destroy": (None, [_vp]),
    "magma_comm_abort": (None, [_vp]),
    "magma_comm_size": (None, [_vp, C.POINTER(_i32)]),
    "magma_comm_rank": (None, [_vp, C.POINTER(_i32)]),
    "magma_comm_check": (None, [_vp]),
    "magma_allreduce": (None, [_vp, _vp, _i64, _i32, _i32, _vp, _vp]),
    "magma_reduce_scatter": (None, [_vp, _vp, _i64, _i32, _i32, _vp, _vp]),
    "magma_all_gather": (None, [_vp, _vp, _i64, _i32, _vp, _vp]),
    "magma_group_start": (None, []),
    "magma_group_end": (None, []),
    "magma_event_create": (None, [C.POINTER(_vp), _i32]),
    "magma_event_destroy": (None, [_vp]),
    "magma_event_record": (None, [_vp, _vp]),
    "magma_stream_wait_event": (None, [_vp, _vp]),
    "magma_event_synchronize": (None, [_vp]),
    "magma_event_query": (None, [_vp, C.POINTER(_i32)]),
    "magma_event_elapsed_ms": (None, [_vp, _vp, C.POINTER(_f)]),
    "magma_scale": (None, [_vp, _i64, _f, _vp]),
}

# Kernel launches one successful call of each op makes (for launch accounting).
KERNELS_PER_CALL = {
    "magma_layernorm_fwd": 1, "magma_layernorm_bwd": 2, "magma_layernorm_bwd_noalloc": 2,
    "magma_layernorm_bwd_residual": 2,
    "magma_gemm": 1,
    "magma_attention_fwd": 1, "magma_attention_bwd": 3, "magma_adam_step": 1,
    "magma_adam_step_multi": 1, "magma_embedding_fwd": 1, "magma_embedding_bwd": 2,
    "magma_grad_norm": 2, "magma_adam_step_clipped": 1, "magma_lr_warmup_cosine": 0,
    "magma_embedding_bwd_deterministic": 4,
    "magma_cross_entropy_fwd_bwd": 1,
    "magma_cross_entropy_fwd_bwd_rowstats": 1, "magma_reduce_sum": 1, "magma_gelu_fwd": 1,
    "magma_gelu_bwd": 1, "magma_relu_fwd": 1, "magma_relu_bwd": 1, "magma_bias_grad": 2,
    "magma_convert": 1, "magma_scale": 1, "magma_mse_fwd_bwd": 1, "magma_memset": 0,
    # collectives run NCCL's kernels, not this library's
    "magma_allreduce": 0, "magma_reduce_scatter": 0, "magma_all_gather": 0,
    "magma_grad_sumsq": 2, "magma_grad_norm_combine": 1,
}

_lib = None
_lock = threading.Lock()


def load() -> C.CDLL:
    """Loads libmagma_cuda.so (raises if it is missing; there is no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with `python -m magma_b200.build`")
            L = C.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = None if res == "void" else (C.c_int32 if res is None else res)
                fn.argtypes = args
            _lib = L
    return _lib


def call(name: str, *args) -> None:
    """Calls a status-returning entry point and raises MagmaError on failure."""
    L = load()
    L.magma_clear_last_error_message()
    status = getattr(L, name)(*args)
    if status != OK:
        msg = L.magma_get_last_error_message()
        raise MagmaError(name, int(status), msg.decode() if msg else None)


def query(name: str, *args) -> int:
    """Calls a size-returning entry point (``*_workspace_size``)."""
    return int(getattr(load(), name)(*args))


def declared_symbols(header: Path | None = None) -> list[str]:
    """Names of every function include/magma_cuda.h declares."""
    import re
    header = header or PKG.parent / "include" / "magma_cuda.h"
    text = header.read_text()
    return sorted(set(re.findall(r"MAGMA_API\s+[\w\s\*]+?\b(magma_\w+)\s*\(", text)))
