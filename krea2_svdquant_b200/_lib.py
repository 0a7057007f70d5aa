"""ctypes binding of ``libsvdq_b200.so`` (the C ABI in ``include/svdq_b200.h``).

The library is loaded from this package directory.  There is no fallback:
if it is missing or fails to load, every op raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libsvdq_b200.so")

_lock = threading.Lock()
_lib = None

c_void_p = ctypes.c_void_p
c_int = ctypes.c_int
c_int64 = ctypes.c_int64

class GemmProblem(ctypes.Structure):
    """``svdq_gemm_problem`` of include/svdq_b200.h: one GEMM of ``svdq_linear_gemm_group``."""
    _fields_ = [("a16", c_void_p), ("w16", c_void_p), ("mid_hl", c_void_p), ("up_hl", c_void_p),
                ("bias", c_void_p), ("epilogue", c_int), ("aux", c_void_p), ("ld_aux", c_int64),
                ("out", c_void_p), ("ldo", c_int64), ("N", c_int)]


# name -> (argtypes, restype) for every entry point of include/svdq_b200.h
SIGNATURES = {
    "svdq_last_error": ([], ctypes.c_char_p),
    "svdq_version": ([], ctypes.c_char_p),
    "svdq_device_error": ([ctypes.POINTER(c_int), c_int], c_int),
    "svdq_selftest_bounded_wait": ([c_int, c_void_p], c_int),
    "svdq_selftest_epilogue_act": ([c_int, c_void_p, c_void_p, c_int, c_void_p], c_int),
    "svdq_act_quant_workspace_bytes": ([c_int, c_int, c_int, c_int], ctypes.c_size_t),
    "svdq_act_quant": ([c_void_p, c_int64, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int,
                        c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int,
                        c_void_p, ctypes.c_size_t, c_void_p], c_int),
    "svdq_act_quant_i8": ([c_void_p, c_int64, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int,
                           c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_int64, c_void_p, c_int,
                           c_void_p, ctypes.c_size_t, c_void_p], c_int),
    "svdq_act_quant_noalloc_scratch_bytes": ([], ctypes.c_size_t),
    "svdq_act_quant_noalloc": ([c_void_p, c_int64, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int,
                                c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int,
                                c_void_p], c_int),
    "svdq_w4a16_prep": ([c_void_p, c_int64, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int,
                         c_int, c_int, c_int, c_void_p, c_void_p, c_int, c_void_p, ctypes.c_size_t,
                         c_void_p], c_int),
    "svdq_prefetcher_create": ([c_int, c_int, ctypes.POINTER(c_void_p)], c_int),
    "svdq_prefetcher_copy_stream": ([c_void_p, ctypes.POINTER(c_void_p)], c_int),
    "svdq_prefetch_begin": ([c_void_p, c_int, c_void_p, c_void_p, ctypes.c_size_t], c_int),
    "svdq_prefetch_commit": ([c_void_p, c_int], c_int),
    "svdq_prefetch_wait": ([c_void_p, c_int, c_void_p, c_int], c_int),
    "svdq_prefetch_release": ([c_void_p, c_int, c_void_p], c_int),
    "svdq_prefetcher_sync": ([c_void_p, c_int], c_int),
    "svdq_prefetcher_destroy": ([c_void_p], c_int),
    "svdq_quantize_weight": ([c_void_p, c_int64, c_int, c_int, c_int, c_void_p, c_void_p, c_int, c_void_p], c_int),
    "svdq_repack_weight": ([c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p], c_int),
    "svdq_build_up_hl": ([c_void_p, c_int, c_void_p, c_int, c_int, c_void_p, c_int, c_void_p], c_int),
    "svdq_linear_gemm": ([c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int,
                          c_int64, c_int, c_int, c_int, c_void_p], c_int),
    "svdq_linear_gemm_workspace_bytes": ([], ctypes.c_size_t),
    "svdq_linear_gemm_ws": ([c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int,
                             c_int64, c_int, c_int, c_int, c_void_p, ctypes.c_size_t, c_void_p], c_int),
    "svdq_linear_gemm_epi": ([c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int64,
                              c_void_p, c_int, c_int64, c_int, c_int, c_int, c_void_p, ctypes.c_size_t, c_void_p],
                             c_int),
    "svdq_linear_gemm_small": ([c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int, c_int64,
                                c_int, c_int, c_int, c_void_p], c_int),
    "svdq_linear_gemm_group": ([ctypes.POINTER(GemmProblem), c_int, c_int, c_int, c_int, c_int, c_void_p,
                                ctypes.c_size_t, c_void_p], c_int),
    "svdq_linear_gemm_schedule": ([c_int, c_int, c_int, c_int, c_int, ctypes.POINTER(c_int)], c_int),
    "svdq_linear_gemm_plan": ([c_int, c_int, c_int, c_int, ctypes.POINTER(c_int)], c_int),
    "svdq_prepare_packed": ([c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p,
                             c_void_p], c_int),
    "svdq_packed_gemm": ([c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int,
                          c_int64, c_int, c_int, c_int, c_void_p], c_int),
    "svdq_w4a4_gemm": ([c_void_p, c_void_p, c_int64, c_int, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int,
                        c_void_p, c_void_p, c_int, c_int64, c_int, c_int, c_int, c_void_p], c_int),
    "svdq_packed_gemm_plan": ([c_int, c_int, c_int, ctypes.POINTER(c_int)], c_int),
    "svdq_w4a4_gemm_narrow": ([c_void_p, c_void_p, c_int64, c_int, c_void_p, c_void_p, c_int, c_void_p, c_void_p,
                               c_int, c_void_p, c_void_p, c_int, c_int64, c_int, c_int, c_int, c_void_p], c_int),
}

SVDQ_BF16, SVDQ_FP16, SVDQ_FP32 = 0, 1, 2
SVDQ_EPI_NONE, SVDQ_EPI_ADD, SVDQ_EPI_SIGMOID_MUL, SVDQ_EPI_SILU_MUL = 0, 1, 2, 3
STATUS_NAMES = {0: "SVDQ_OK", 1: "SVDQ_ERR_INVALID_ARGUMENT", 2: "SVDQ_ERR_UNSUPPORTED",
                3: "SVDQ_ERR_CUDA", 4: "SVDQ_ERR_TIMEOUT", 5: "SVDQ_ERR_DEVICE_WAIT"}


class SVDQError(RuntimeError):
    """A C-ABI entry point returned a non-zero status."""

    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


def lib() -> ctypes.CDLL:
    """Load (once) and return the library; raises if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m krea2_svdquant_b200.build` "
                    "(there is no non-CUDA fallback)")
            handle = ctypes.CDLL(LIB_PATH)
            for name, (argtypes, restype) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.argtypes = argtypes
                fn.restype = restype
            _lib = handle
    return _lib


def check(status: int) -> None:
    if status != 0:
        raise SVDQError(status, lib().svdq_last_error().decode(errors="replace"))


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))


def device_error(clear: bool = True) -> int:
    """Synchronize and return (and clear) the library's device-side wait error word."""
    code = c_int(0)
    check(lib().svdq_device_error(ctypes.byref(code), 1 if clear else 0))
    return code.value


class DeviceWaitError(RuntimeError):
    """A bounded in-kernel wait ran out: the results of the launches since the last check are
    incomplete.  ``code`` is the device error word (see ``svdq_device_error`` in the header)."""

    def __init__(self, code: int, where: str):
        super().__init__(f"device-side wait error 0x{code:x} ({where}): the outputs of the kernels since the "
                         "last check are incomplete")
        self.code = code


def raise_on_device_error(where: str) -> None:
    """Synchronize, read and clear the device error word; raise :class:`DeviceWaitError` if set."""
    code = device_error(clear=True)
    if code:
        raise DeviceWaitError(code, where)
