"""ctypes binding of ``libspinn_cuda.so`` (declared in ``include/spinn_cuda.h``).

There is no fallback: if the CUDA library is missing or fails to load, every entry point
raises.  Build it with ``python -m spinn_b200.build``.
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libspinn_cuda.so")

# Status codes (include/spinn_cuda.h)
OK, EINVAL, ENOMEM, ECUDA, EUNSUPPORTED, ETIMEOUT, EFORMAT, ESTATE = 0, -1, -2, -3, -4, -5, -6, -7
PLAN_NO_GRAPH, PLAN_PROFILE, PLAN_NO_ROUND, PLAN_WINOGRAD, PLAN_KEEP, PLAN_NO_FUSE = 1, 2, 4, 8, 16, 32

# ENNF operator codes (SPINN/ennf_op_types.h:79,134,135)
OP_CONV, OP_GEMM, OP_MATMUL = 60, 160, 161


class SpinnTensor(ctypes.Structure):
    """The reference's runtime tensor record (``SPINN/run_time/spinn_runtime.h:25-40``), 72 bytes."""

    _fields_ = [
        ("id", ctypes.c_uint16),
        ("dtype", ctypes.c_uint8),
        ("ndim", ctypes.c_uint8),
        ("dims", ctypes.c_uint32 * 8),
        ("elem_count", ctypes.c_uint32),
        ("is_weight", ctypes.c_uint8),
        ("ref_count", ctypes.c_uint8),
        ("size", ctypes.c_uint32),
        ("offset", ctypes.c_uint32),
        ("data", ctypes.c_void_p),
        ("packed_data", ctypes.c_void_p),
    ]


assert ctypes.sizeof(SpinnTensor) == 72

SpinnOpKernel = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.POINTER(ctypes.POINTER(SpinnTensor)), ctypes.c_int,
                                 ctypes.c_void_p, ctypes.c_uint16,
                                 ctypes.POINTER(ctypes.POINTER(SpinnTensor)), ctypes.c_int)
RegisterFn = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_uint16, SpinnOpKernel)

_lib = None
_lock = threading.Lock()

# name -> (restype, argtypes)
_SIGS = {
    "spinn_cuda_init": (ctypes.c_int, [ctypes.c_int, ctypes.c_size_t]),
    "spinn_cuda_sync": (ctypes.c_int, []),
    "spinn_cuda_shutdown": (None, []),
    "spinn_cuda_last_error": (ctypes.c_char_p, []),
    "spinn_cuda_register": (ctypes.c_int, [ctypes.c_void_p]),
    "spinn_cuda_conv2d": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_uint16,
                                         ctypes.c_void_p, ctypes.c_int]),
    "spinn_cuda_gemm": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_uint16,
                                       ctypes.c_void_p, ctypes.c_int]),
    "spinn_cuda_matmul": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_uint16,
                                         ctypes.c_void_p, ctypes.c_int]),
    "spinn_cuda_conv2d_noalloc": (ctypes.c_int, [ctypes.c_void_p] * 5 + [ctypes.c_int] * 12 + [ctypes.c_void_p]),
    "spinn_cuda_load": (ctypes.c_void_p, [ctypes.c_char_p]),
    "spinn_cuda_load_buffer": (ctypes.c_void_p, [ctypes.c_void_p, ctypes.c_size_t]),
    "spinn_cuda_plan": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_uint64, ctypes.c_int]),
    "spinn_cuda_run": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "spinn_cuda_run_device": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "spinn_cuda_submit": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "spinn_cuda_selftest_wait_expiry": (ctypes.c_int, [ctypes.c_uint64]),
    "spinn_cuda_selftest_flag_wait_expiry": (ctypes.c_int, [ctypes.c_uint64]),
    "spinn_cuda_wait": (ctypes.c_int, [ctypes.c_void_p]),
    "spinn_cuda_run_profiled": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "spinn_cuda_io_ptr": (ctypes.c_void_p, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                           ctypes.POINTER(ctypes.c_size_t)]),
    "spinn_cuda_io_count": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "spinn_cuda_io_dtype": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]),
    "spinn_cuda_copy_output": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t]),
    "spinn_cuda_copy_tensor": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                              ctypes.c_void_p, ctypes.c_size_t]),
    "spinn_cuda_io_dims": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                          ctypes.POINTER(ctypes.c_uint32)]),
    "spinn_cuda_plan_info": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint64),
                                            ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_int),
                                            ctypes.POINTER(ctypes.c_int)]),
    "spinn_cuda_profile": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int),
                                          ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_double),
                                          ctypes.c_int]),
    "spinn_cuda_step_kind": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "spinn_cuda_free": (None, [ctypes.c_void_p]),
    "spinn_cuda_host_alloc": (ctypes.c_void_p, [ctypes.c_size_t]),
    "spinn_cuda_host_free": (None, [ctypes.c_void_p]),
    "spinn_cuda_version": (ctypes.c_char_p, []),
    "spinn_cuda_stat_streamk_launches": (ctypes.c_uint64, []),
    "spinn_cuda_diag_tile_plan": (ctypes.c_int, [ctypes.c_int] * 8 + [ctypes.POINTER(ctypes.c_int)]),
    "spinn_cuda_diag_streamk_piece": (ctypes.c_int, [ctypes.c_int] * 5 + [ctypes.POINTER(ctypes.c_int)]),
    "spinn_cuda_diag_streamk_contributes": (ctypes.c_int, [ctypes.c_int] * 5),
}


class SpinnCudaError(RuntimeError):
    def __init__(self, code: int, where: str, msg: str):
        super().__init__(f"{where} failed ({code}): {msg}")
        self.code = code


def lib() -> ctypes.CDLL:
    """Loads libspinn_cuda.so once (raises if it is absent)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(f"{LIB_PATH} is missing; build it with `python -m spinn_b200.build`")
            L = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_LOCAL)
            for name, (res, args) in _SIGS.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def declared_symbols():
    return sorted(_SIGS)


def last_error() -> str:
    return (lib().spinn_cuda_last_error() or b"").decode(errors="replace")


def check(rc: int, where: str) -> int:
    if rc < 0:
        raise SpinnCudaError(rc, where, last_error())
    return rc
