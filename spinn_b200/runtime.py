"""Host-side API mirroring SPINN's operator and runtime interfaces.

* Operator level -- :func:`conv2d`, :func:`gemm`, :func:`matmul` call the C-ABI drop-in
  kernels with the reference's argument conventions (``SpinnTensor`` records, ENNF
  parameter blocks; ``SPINN/run_time/ops/conv/conv2d.c``, ``ops/mm/gemm.c``,
  ``ops/mm/matmul.c``).  Arrays may be NumPy (host memory, like the reference arena) or
  CUDA torch tensors (device memory).
* Model level -- :class:`Model` wraps ``spinn_cuda_load / _plan / _run / _free``, the
  device-resident counterpart of ``spinn_load / spinn_plan / spinn_run / spinn_free``
  (``SPINN/run_time/spinn_runtime.h:107-133``).
"""
from __future__ import annotations

import ctypes
import struct
from typing import List, Optional, Sequence

import numpy as np

from . import lib as _L
from .lib import SpinnTensor, check, lib

CONV_PARAMS_FMT = "<4H4H8H4HHBB"   # ENNF_ConvParams (SPINN/ennf_op_params.h:23-31)
GEMM_PARAMS_FMT = "<ffBB2x"        # ENNF_GemmParams (SPINN/ennf_op_params.h:134-140)


def conv_params(kernel=(0, 0), strides=(1, 1), pads=(0, 0, 0, 0), dilations=(1, 1), group=1,
                auto_pad=0, fused_act=0) -> bytes:
    """Packs an ``ENNF_ConvParams`` block; ``fused_act`` goes into ``reserved``."""
    def pad(v, n):
        v = list(v)[:n]
        return v + [0] * (n - len(v))
    return struct.pack(CONV_PARAMS_FMT, *pad(kernel, 4), *pad(strides, 4), *pad(pads, 8),
                       *pad(dilations, 4), group, auto_pad, fused_act)


def gemm_params(alpha=1.0, beta=1.0, trans_a=0, trans_b=0) -> bytes:
    return struct.pack(GEMM_PARAMS_FMT, alpha, beta, trans_a, trans_b)


class _Arg:
    """A SpinnTensor record over a NumPy array (host) or a CUDA torch tensor (device)."""

    def __init__(self, arr, is_weight: bool = False, tid: int = 0):
        self.arr = arr
        t = SpinnTensor()
        shape = tuple(arr.shape)
        if len(shape) > 8:
            raise ValueError("at most 8 dimensions")
        t.id = tid
        t.dtype = 1
        t.ndim = len(shape)
        for i, d in enumerate(shape):
            t.dims[i] = int(d)
        n = int(np.prod(shape)) if shape else 1
        t.elem_count = n
        t.is_weight = 1 if is_weight else 0
        t.size = n * 4
        if isinstance(arr, np.ndarray):
            if arr.dtype != np.float32 or not arr.flags["C_CONTIGUOUS"]:
                raise TypeError("host arrays must be C-contiguous float32")
            t.data = arr.ctypes.data
        else:  # torch tensor
            import torch
            if arr.dtype != torch.float32 or not arr.is_contiguous():
                raise TypeError("torch tensors must be contiguous float32")
            t.data = arr.data_ptr()
        self.rec = t


def _call(fn_name: str, ins: Sequence[_Arg], outs: Sequence[_Arg], params: bytes) -> None:
    n_in, n_out = len(ins), len(outs)
    in_arr = (ctypes.POINTER(SpinnTensor) * n_in)(*[ctypes.pointer(a.rec) for a in ins])
    out_arr = (ctypes.POINTER(SpinnTensor) * n_out)(*[ctypes.pointer(a.rec) for a in outs])
    pbuf = ctypes.create_string_buffer(params, len(params)) if params else None
    rc = getattr(lib(), fn_name)(ctypes.cast(in_arr, ctypes.c_void_p), n_in,
                                 ctypes.cast(pbuf, ctypes.c_void_p) if pbuf else None, len(params),
                                 ctypes.cast(out_arr, ctypes.c_void_p), n_out)
    check(rc, fn_name)


def init(device: int = 0, scratch_bytes: int = 0) -> None:
    check(lib().spinn_cuda_init(device, scratch_bytes), "spinn_cuda_init")


def sync() -> None:
    check(lib().spinn_cuda_sync(), "spinn_cuda_sync")


def shutdown() -> None:
    lib().spinn_cuda_shutdown()


def conv2d(x, w, y, bias=None, residual=None, params: bytes = b"") -> None:
    """``op_conv2d`` semantics: inputs [X, W, (B), (R)], residual last when the fused act is 4/5."""
    ins = [_Arg(x), _Arg(w, True)]
    if bias is not None:
        ins.append(_Arg(bias, True))
    if residual is not None:
        ins.append(_Arg(residual))
    _call("spinn_cuda_conv2d", ins, [_Arg(y)], params or conv_params())


def gemm(a, b, y, c=None, params: bytes = b"", b_is_weight: bool = True) -> None:
    ins = [_Arg(a), _Arg(b, b_is_weight)]
    if c is not None:
        ins.append(_Arg(c, True))
    _call("spinn_cuda_gemm", ins, [_Arg(y)], params or gemm_params())


def matmul(a, b, y) -> None:
    _call("spinn_cuda_matmul", [_Arg(a), _Arg(b)], [_Arg(y)], b"")


class Model:
    """A ``.ennf`` model planned on one GPU (load -> plan -> run)."""

    def __init__(self, source, device: int = 0, max_arena_bytes: int = 0, flags: int = 0):
        L = lib()
        if isinstance(source, (bytes, bytearray, memoryview)):
            buf = bytes(source)
            self._h = L.spinn_cuda_load_buffer(buf, len(buf))
        else:
            self._h = L.spinn_cuda_load(str(source).encode())
        if not self._h:
            raise _L.SpinnCudaError(_L.EFORMAT, "spinn_cuda_load", _L.last_error())
        self.device = device
        self.flags = flags
        try:
            check(L.spinn_cuda_plan(self._h, device, max_arena_bytes, flags), "spinn_cuda_plan")
        except Exception:
            L.spinn_cuda_free(self._h)
            self._h = None
            raise

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().spinn_cuda_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def io_dims(self, is_output: bool, index: int = 0) -> List[int]:
        dims = (ctypes.c_uint32 * 8)()
        nd = check(lib().spinn_cuda_io_dims(self._h, int(is_output), index, dims), "spinn_cuda_io_dims")
        return [int(dims[i]) for i in range(nd)]

    def io_count(self, is_output: bool) -> int:
        return check(lib().spinn_cuda_io_count(self._h, int(is_output)), "spinn_cuda_io_count")

    def io_ptr(self, is_output: bool, index: int = 0):
        n = ctypes.c_size_t(0)
        p = lib().spinn_cuda_io_ptr(self._h, int(is_output), index, ctypes.byref(n))
        if not p:
            raise _L.SpinnCudaError(_L.ESTATE, "spinn_cuda_io_ptr", "no such buffer")
        return p, n.value

    def output(self, index: int) -> np.ndarray:
        """Graph output `index` of the last run, copied to host (fp32 or int64)."""
        dt = np.int64 if check(lib().spinn_cuda_io_dtype(self._h, 1, index), "spinn_cuda_io_dtype") == 7 \
            else np.float32
        out = np.empty(self.io_dims(True, index), dt)
        check(lib().spinn_cuda_copy_output(self._h, index, out.ctypes.data, out.nbytes), "spinn_cuda_copy_output")
        return out

    def tensor(self, tensor_id: int, dims: Sequence[int], first: int = 0, count: Optional[int] = None,
               dtype=np.float32) -> np.ndarray:
        """Items ``first .. first+count-1`` (dim 0) of ENNF tensor `tensor_id` after a run, in the
        .ennf layout (``dims`` as the .ennf declares them; ``spinn_cuda_copy_tensor``).  Any
        activation when planned with ``PLAN_KEEP``, otherwise graph outputs only."""
        count = int(dims[0]) - first if count is None else count
        out = np.empty((count,) + tuple(int(d) for d in dims[1:]), dtype)
        check(lib().spinn_cuda_copy_tensor(self._h, int(tensor_id), int(first), int(count), out.ctypes.data,
                                           out.nbytes), "spinn_cuda_copy_tensor")
        return out

    def run(self, x: np.ndarray, out: Optional[np.ndarray] = None) -> np.ndarray:
        """Host input -> host output 0 (``spinn_run``)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        if out is None:
            out = np.empty(self.io_dims(True, 0), np.float32)
        check(lib().spinn_cuda_run(self._h, x.ctypes.data, out.ctypes.data), "spinn_cuda_run")
        return out

    def run_ptr(self, host_in: int, host_out: int) -> None:
        check(lib().spinn_cuda_run(self._h, host_in, host_out), "spinn_cuda_run")

    def submit_ptr(self, host_in: int, host_out: int) -> None:
        """Queues one run (``spinn_cuda_submit``): host buffers by address, pinned for overlap;
        they must stay untouched until :meth:`wait` returns."""
        check(lib().spinn_cuda_submit(self._h, host_in or None, host_out or None), "spinn_cuda_submit")

    def wait(self) -> None:
        """Waits for every submitted run (``spinn_cuda_wait``)."""
        check(lib().spinn_cuda_wait(self._h), "spinn_cuda_wait")

    def run_device(self, stream: int = 0) -> None:
        check(lib().spinn_cuda_run_device(self._h, stream or None), "spinn_cuda_run_device")

    def run_profiled(self, stream: int = 0) -> None:
        """One run with per-step device timing (plan with PLAN_PROFILE); synchronous."""
        check(lib().spinn_cuda_run_profiled(self._h, stream or None), "spinn_cuda_run_profiled")

    def plan_info(self) -> dict:
        a, w = ctypes.c_uint64(0), ctypes.c_uint64(0)
        s, k = ctypes.c_int(0), ctypes.c_int(0)
        check(lib().spinn_cuda_plan_info(self._h, ctypes.byref(a), ctypes.byref(w), ctypes.byref(s),
                                         ctypes.byref(k)), "spinn_cuda_plan_info")
        return {"arena_bytes": a.value, "weight_bytes": w.value, "steps": s.value, "kernels": k.value}

    def step_kinds(self) -> List[int]:
        n = self.plan_info()["steps"]
        return [lib().spinn_cuda_step_kind(self._h, i) for i in range(n)]

    def profile(self):
        """(op_type, ms, flops) per step of the last run; plan with PLAN_PROFILE."""
        n = self.plan_info()["steps"]
        ops = (ctypes.c_int * n)()
        ms = (ctypes.c_float * n)()
        fl = (ctypes.c_double * n)()
        k = check(lib().spinn_cuda_profile(self._h, ops, ms, fl, n), "spinn_cuda_profile")
        return [(ops[i], ms[i], fl[i]) for i in range(k)]
