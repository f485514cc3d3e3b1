"""CPU oracle for SPINN's dense-contraction hot path (TEST INFRASTRUCTURE).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg use this module,
and only as the checker / the timed CPU baseline.  Two implementations:

* :class:`RefOracle` -- the reference's own operators and runtime, compiled unmodified from
  the reference sources into ``oracle/_ref/libspinn_ref.so`` by ``oracle/Makefile``
  ("O-fix": the group==1 conv epilogue restored by ``ref_shim.c``; ``fix=False`` gives the
  shipped behaviour).  Built in the development container; the built file travels with
  the tree.
* :class:`PortOracle` -- this repo's plain-C restatement (``oracle/spinn_oracle.c``), built
  into ``oracle/_build/liboracle_port.so``; always buildable.

Both run ``.ennf`` models: the reference through its own ``spinn_load/plan/run``, the port
through a node loop over its operators (:meth:`PortOracle.run_model`).
"""
from __future__ import annotations

import ctypes
import os
import struct
import subprocess
import sys
import tempfile
from typing import Dict, Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from spinn_b200 import ennf  # noqa: E402
from spinn_b200.lib import SpinnTensor  # noqa: E402

REF_LIB = os.path.join(HERE, "_ref", "libspinn_ref.so")
REF_CONVERTER = os.path.join(HERE, "_ref", "onnx2ennf")
PORT_LIB = os.path.join(HERE, "_build", "liboracle_port.so")

_f32p = ctypes.POINTER(ctypes.c_float)


def _fp(a: Optional[np.ndarray]):
    return a.ctypes.data_as(_f32p) if a is not None else None


def reference_dir() -> Optional[str]:
    """The reference's ``SPINN/`` source directory: ``$REF_DIR`` when set, else a ``reference``
    checkout beside this repository; None when neither exists (the GPU box has only the
    prebuilt ``_ref`` files)."""
    cands = [os.environ.get("REF_DIR"), os.path.join(os.path.dirname(ROOT), "reference", "SPINN")]
    for c in cands:
        if c and os.path.isfile(os.path.join(c, "run_time", "spinn_runtime.c")):
            return os.path.abspath(c)
    return None


def build(ref: bool = True) -> None:
    """Builds the port (always) and the reference library (when the reference tree exists)."""
    targets = ["port"]
    rd = reference_dir() if ref else None
    if rd:
        targets.append("ref")
    subprocess.run(["make", "-s", "-C", HERE] + targets + ([f"REF_DIR={rd}"] if rd else []), check=True)


def ref_available() -> bool:
    return os.path.exists(REF_LIB)


class _T:
    """SpinnTensor over a host NumPy array."""

    def __init__(self, arr: np.ndarray, is_weight=False):
        self.arr = np.ascontiguousarray(arr, dtype=np.float32)
        t = SpinnTensor()
        t.dtype = 1
        t.ndim = self.arr.ndim
        for i, d in enumerate(self.arr.shape):
            t.dims[i] = d
        t.elem_count = self.arr.size
        t.size = self.arr.size * 4
        t.is_weight = 1 if is_weight else 0
        t.data = self.arr.ctypes.data
        self.rec = t


def _op_call(fn, ins, outs, params: bytes) -> int:
    in_arr = (ctypes.POINTER(SpinnTensor) * len(ins))(*[ctypes.pointer(t.rec) for t in ins])
    out_arr = (ctypes.POINTER(SpinnTensor) * len(outs))(*[ctypes.pointer(t.rec) for t in outs])
    pbuf = ctypes.create_string_buffer(params, len(params)) if params else None
    return fn(in_arr, len(ins), pbuf, len(params), out_arr, len(outs))


class RefOracle:
    """The reference implementation (oracle/_ref/libspinn_ref.so)."""

    def __init__(self, fix: bool = True, threads: Optional[int] = None):
        if not ref_available():
            raise FileNotFoundError(f"{REF_LIB} not built (make -C oracle ref)")
        L = ctypes.CDLL(REF_LIB, mode=ctypes.RTLD_LOCAL)
        self.L = L
        L.spinn_load.restype = ctypes.c_void_p
        L.spinn_load.argtypes = [ctypes.c_char_p]
        L.spinn_plan.argtypes = [ctypes.c_void_p, ctypes.c_uint32]
        L.spinn_run.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        L.spinn_free.argtypes = [ctypes.c_void_p]
        for n in ("spinn_oracle_num_outputs", "spinn_oracle_num_inputs", "spinn_oracle_num_nodes"):
            getattr(L, n).argtypes = [ctypes.c_void_p]
        L.spinn_oracle_output_id.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.spinn_oracle_input_id.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.spinn_oracle_tensor_size.restype = ctypes.c_uint32
        L.spinn_oracle_tensor_size.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.spinn_oracle_copy_tensor.restype = ctypes.c_long
        L.spinn_oracle_copy_tensor.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t]
        L.spinn_oracle_arena_bytes.restype = ctypes.c_size_t
        L.spinn_oracle_arena_bytes.argtypes = [ctypes.c_void_p]
        L.spinn_oracle_sizeof_tensor.restype = ctypes.c_size_t
        L.winograd_pack_weight.restype = ctypes.c_void_p
        L.winograd_pack_weight.argtypes = [_f32p, ctypes.c_int, ctypes.c_int]
        L.winograd_conv_3x3.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                        ctypes.c_int, _f32p, ctypes.c_int, ctypes.c_int, _f32p, ctypes.c_int,
                                        ctypes.c_int, ctypes.c_int]
        L.sgemm_tiled.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, _f32p, ctypes.c_int,
                                  _f32p, ctypes.c_int, ctypes.c_float, _f32p, ctypes.c_int]
        L.spinn_register_op.argtypes = [ctypes.c_uint16, ctypes.c_void_p]
        self.libc = ctypes.CDLL(None)
        self.libc.free.argtypes = [ctypes.c_void_p]
        self.set_fix(fix)
        if threads:
            L.spinn_oracle_set_threads(int(threads))

    def set_fix(self, on: bool) -> None:
        self.L.spinn_oracle_set_fix(1 if on else 0)

    def set_threads(self, n: int) -> None:
        self.L.spinn_oracle_set_threads(int(n))

    def max_threads(self) -> int:
        return self.L.spinn_oracle_max_threads()

    # ---------------------------------------------------------------- operators
    def conv2d(self, x, w, bias=None, residual=None, params: bytes = b"", out_shape=None) -> np.ndarray:
        ins = [_T(x), _T(w, True)]
        if bias is not None:
            ins.append(_T(bias, True))
        if residual is not None:
            ins.append(_T(residual))
        y = _T(np.zeros(out_shape, np.float32))
        rc = _op_call(self.L.op_conv2d, ins, [y], params)
        if rc != 0:
            raise RuntimeError(f"op_conv2d returned {rc}")
        return y.arr

    def gemm(self, a, b, c=None, params: bytes = b"", out_shape=None) -> np.ndarray:
        ins = [_T(a), _T(b, True)] + ([_T(c, True)] if c is not None else [])
        y = _T(np.zeros(out_shape, np.float32))
        rc = _op_call(self.L.op_gemm, ins, [y], params)
        if rc != 0:
            raise RuntimeError(f"op_gemm returned {rc}")
        return y.arr

    def matmul(self, a, b, out_shape) -> np.ndarray:
        y = _T(np.zeros(out_shape, np.float32))
        rc = _op_call(self.L.op_matmul, [_T(a), _T(b)], [y], b"")
        if rc != 0:
            raise RuntimeError(f"op_matmul returned {rc}")
        return y.arr

    def winograd_f23(self, x, w, bias, ph, pw, oh, ow, relu) -> np.ndarray:
        n, c, h, wd = x.shape
        oc = w.shape[0]
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        u = self.L.winograd_pack_weight(_fp(w), oc, c)
        y = np.zeros((n, oc, oh, ow), np.float32)
        b = np.ascontiguousarray(bias, np.float32) if bias is not None else None
        rc = self.L.winograd_conv_3x3(_fp(x), n, c, h, wd, u, oc, _fp(b), ph, pw, _fp(y), oh, ow, int(relu))
        self.libc.free(u)
        if rc != 0:
            raise RuntimeError(f"winograd_conv_3x3 returned {rc}")
        return y

    # ---------------------------------------------------------------- models
    def run_model(self, path: str, x: np.ndarray, all_outputs: bool = True) -> Dict[int, np.ndarray]:
        """spinn_load -> spinn_plan -> spinn_run; returns {tensor id: output}."""
        L = self.L
        ctx = L.spinn_load(path.encode())
        if not ctx:
            raise RuntimeError(f"spinn_load({path}) failed")
        try:
            rc = L.spinn_plan(ctx, 0)
            if rc != 0:
                raise RuntimeError(f"spinn_plan returned {rc}")
            x = np.ascontiguousarray(x, np.float32)
            L.spinn_oracle_reset_status()
            L.spinn_run(ctx, x.ctypes.data, None)
            status = L.spinn_oracle_first_status()
            if status != 0:
                raise RuntimeError(f"an operator returned {status} during spinn_run")
            outs = {}
            for i in range(L.spinn_oracle_num_outputs(ctx) if all_outputs else 1):
                tid = L.spinn_oracle_output_id(ctx, i)
                n = L.spinn_oracle_tensor_size(ctx, tid) // 4
                buf = np.empty(n, np.float32)
                if L.spinn_oracle_copy_tensor(ctx, tid, buf.ctypes.data, buf.nbytes) < 0:
                    raise RuntimeError(f"output tensor {tid} has no data")
                outs[tid] = buf
            return outs
        finally:
            L.spinn_free(ctx)

    def time_model(self, path: str, x: np.ndarray, steps: int, warmup: int = 1):
        """Seconds per spinn_run (wall clock, CLOCK_MONOTONIC via time.perf_counter)."""
        import time
        L = self.L
        ctx = L.spinn_load(path.encode())
        if not ctx or L.spinn_plan(ctx, 0) != 0:
            raise RuntimeError("spinn_load/plan failed")
        x = np.ascontiguousarray(x, np.float32)
        try:
            for _ in range(warmup):
                L.spinn_run(ctx, x.ctypes.data, None)
            ts = []
            for _ in range(steps):
                t0 = time.perf_counter()
                L.spinn_run(ctx, x.ctypes.data, None)
                ts.append(time.perf_counter() - t0)
            return ts
        finally:
            L.spinn_free(ctx)

    def register_op_fn(self):
        """Address of the shim's spinn_register_op (for spinn_cuda_register)."""
        return ctypes.cast(self.L.spinn_register_op, ctypes.c_void_p).value

    def clear_overrides(self) -> None:
        self.L.spinn_oracle_clear_overrides()


def convert_with_reference(onnx_bytes: bytes) -> bytes:
    """Runs the reference converter (oracle/_ref/onnx2ennf) on an ONNX image."""
    with tempfile.TemporaryDirectory() as d:
        src, dst = os.path.join(d, "m.onnx"), os.path.join(d, "m.ennf")
        with open(src, "wb") as f:
            f.write(onnx_bytes)
        r = subprocess.run([REF_CONVERTER, src, dst], capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"onnx2ennf failed: {r.stdout[-2000:]} {r.stderr[-2000:]}")
        with open(dst, "rb") as f:
            return f.read()


class PortOracle:
    """This repo's C restatement of the hot path (oracle/spinn_oracle.c)."""

    def __init__(self):
        if not os.path.exists(PORT_LIB):
            build(ref=False)
        L = ctypes.CDLL(PORT_LIB, mode=ctypes.RTLD_LOCAL)
        self.L = L
        i = ctypes.c_int
        L.oracle_conv2d.argtypes = [_f32p, i, i, i, i, _f32p, i, i, i, i, i, i, i, i, i, i, _f32p, i, _f32p, _f32p, i, i]
        L.oracle_gemm.argtypes = [_f32p, _f32p, _f32p, ctypes.c_long, _f32p, i, i, i, i, i, ctypes.c_float,
                                  ctypes.c_float, i]
        L.oracle_matmul.argtypes = [_f32p, _f32p, _f32p, i, i, i, i, i]
        L.oracle_winograd_f23_pack.argtypes = [_f32p, i, i, _f32p]
        L.oracle_winograd_f23.argtypes = [_f32p, i, i, i, i, _f32p, i, _f32p, i, i, _f32p, i, i, i]
        L.oracle_winograd_f43_pack.argtypes = [_f32p, i, i, _f32p]
        L.oracle_winograd_f43.argtypes = [_f32p, i, i, i, i, _f32p, i, _f32p, i, _f32p, i, i, _f32p, i, i]
        L.oracle_maxpool.argtypes = [_f32p, i, i, i, i, i, i, i, i, i, i, _f32p, i, i]
        L.oracle_global_avg_pool.argtypes = [_f32p, i, i, i, _f32p]
        L.oracle_add.argtypes = [_f32p, ctypes.c_long, _f32p, ctypes.c_long, _f32p, ctypes.c_long]
        L.oracle_relu.argtypes = [_f32p, _f32p, ctypes.c_long]
        L.oracle_sigmoid.argtypes = [_f32p, _f32p, ctypes.c_long]
        L.oracle_batch_norm.argtypes = [_f32p, i, i, i, _f32p, _f32p, _f32p, _f32p, ctypes.c_float, _f32p]

    def conv2d(self, x, w, bias=None, residual=None, stride=(1, 1), pads=(0, 0), dil=(1, 1), group=1, act=0,
               out_hw=None) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        n, c, h, wd = x.shape
        oc, kc, kh, kw = w.shape
        if out_hw is None:
            out_hw = ((h + 2 * pads[0] - ((kh - 1) * dil[0] + 1)) // stride[0] + 1,
                      (wd + 2 * pads[1] - ((kw - 1) * dil[1] + 1)) // stride[1] + 1)
        y = np.zeros((n, oc) + tuple(out_hw), np.float32)
        b = np.ascontiguousarray(bias, np.float32) if bias is not None else None
        r = np.ascontiguousarray(residual, np.float32) if residual is not None else None
        rc = self.L.oracle_conv2d(_fp(x), n, c, h, wd, _fp(w), oc, kh, kw, stride[0], stride[1], pads[0], pads[1],
                                  dil[0], dil[1], group, _fp(b), act, _fp(r), _fp(y), out_hw[0], out_hw[1])
        if rc != 0:
            raise RuntimeError("oracle_conv2d failed")
        return y

    def gemm(self, a, b, c=None, m=0, n=0, k=0, trans_a=0, trans_b=0, alpha=1.0, beta=1.0, ref_quirk=0):
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        cc = np.ascontiguousarray(c, np.float32) if c is not None else None
        y = np.zeros((m, n), np.float32)
        self.L.oracle_gemm(_fp(a), _fp(b), _fp(cc), cc.size if cc is not None else 0, _fp(y), m, n, k, trans_a, trans_b,
                           alpha, beta, ref_quirk)
        return y

    def matmul(self, a, b) -> np.ndarray:
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        m, k = a.shape[-2:]
        n = b.shape[-1]
        batch = int(np.prod(a.shape[:-2])) if a.ndim > 2 else 1
        b_batch = int(np.prod(b.shape[:-2])) if b.ndim > 2 else 0
        y = np.zeros(a.shape[:-2] + (m, n), np.float32)
        if self.L.oracle_matmul(_fp(a), _fp(b), _fp(y), batch, b_batch, m, n, k) != 0:
            raise RuntimeError("oracle_matmul: batch mismatch")
        return y

    def winograd_f23(self, x, w, bias, ph, pw, oh, ow, relu) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        n, c, h, wd = x.shape
        oc = w.shape[0]
        u = np.zeros(16 * oc * c, np.float32)
        self.L.oracle_winograd_f23_pack(_fp(w), oc, c, _fp(u))
        y = np.zeros((n, oc, oh, ow), np.float32)
        b = np.ascontiguousarray(bias, np.float32) if bias is not None else None
        if self.L.oracle_winograd_f23(_fp(x), n, c, h, wd, _fp(u), oc, _fp(b), ph, pw, _fp(y), oh, ow, int(relu)) != 0:
            raise RuntimeError("oracle_winograd_f23 declined the shape")
        return y

    def winograd_f43_weights(self, w) -> np.ndarray:
        w = np.ascontiguousarray(w, np.float32)
        oc, c = w.shape[:2]
        u = np.zeros((36, oc, c), np.float32)
        self.L.oracle_winograd_f43_pack(_fp(w), oc, c, _fp(u))
        return u

    def winograd_f43(self, x, w, bias=None, act=0, residual=None, ph=1, pw=1) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        n, c, h, wd = x.shape
        oc = w.shape[0]
        u = self.winograd_f43_weights(w)
        oh, ow = h + 2 * ph - 2, wd + 2 * pw - 2
        y = np.zeros((n, oc, oh, ow), np.float32)
        b = np.ascontiguousarray(bias, np.float32) if bias is not None else None
        r = np.ascontiguousarray(residual, np.float32) if residual is not None else None
        self.L.oracle_winograd_f43(_fp(x), n, c, h, wd, _fp(u), oc, _fp(b), act, _fp(r), ph, pw, _fp(y), oh, ow)
        return y

    # ---------------------------------------------------------------- model runner
    @staticmethod
    def topk(x: np.ndarray, k: int):
        """TopK as SPINN/run_time/ops/tensor/topk.c:20-87: last axis, k clamped to its length,
        values descending; equal values keep ascending index order (the reference's qsort is
        glibc's merge sort, stable for its comparator, which treats -0.0 and +0.0 as equal)."""
        x = np.asarray(x, np.float32)
        n = x.shape[-1]
        k = max(0, min(k, n))
        rows = x.reshape(-1, n)
        key = np.where(rows == 0, np.float32(0), rows)        # -0.0 and +0.0 tie
        order = np.argsort(-key.astype(np.float64), axis=1, kind="stable")[:, :k]
        v = np.take_along_axis(rows, order, axis=1)
        return v.reshape(x.shape[:-1] + (k,)), order.astype(np.int64).reshape(x.shape[:-1] + (k,))

    def run_model(self, image: bytes, x: np.ndarray) -> Dict[int, np.ndarray]:
        """Runs an ENNF image node by node over the port operators."""
        m = ennf.read(image)
        vals: Dict[int, np.ndarray] = {}
        vals[m.inputs[0]] = np.ascontiguousarray(x, np.float32).reshape(m.tensors[m.inputs[0]].dims)

        def get(tid):
            if tid in vals:
                return vals[tid]
            if tid in m.weights:
                return np.ascontiguousarray(m.weights[tid])
            raise KeyError(f"tensor {tid} not available")

        for nd in m.nodes:
            op = ennf.OP_NAME.get(nd.op_type)
            out_dims = m.tensors[nd.outputs[0]].dims
            if op == "Conv":
                p = ennf.ConvParams.unpack(nd.params)
                act = p.fused_act
                has_res = act in (4, 5)
                n_real = len(nd.inputs) - (1 if has_res else 0)
                xx, ww = get(nd.inputs[0]), get(nd.inputs[1])
                b = get(nd.inputs[2]) if n_real > 2 else None
                r = get(nd.inputs[-1]) if has_res else None
                kh = p.kernel_shape[0] or ww.shape[2]
                kw = p.kernel_shape[1] or ww.shape[3]
                assert (kh, kw) == tuple(ww.shape[2:])
                y = self.conv2d(xx, ww, b, r, (p.strides[0] or 1, p.strides[1] or 1), (p.pads[0], p.pads[1]),
                                (1, 1), p.group or 1, act, out_dims[2:])
            elif op == "MaxPool":
                v = struct.unpack(ennf.POOL_PARAMS_FMT, nd.params[:48])
                xx = get(nd.inputs[0])
                y = np.zeros(out_dims, np.float32)
                n, c, h, w = xx.shape
                self.L.oracle_maxpool(_fp(xx), n, c, h, w, v[0], v[1], v[4], v[5], v[8], v[9], _fp(y), out_dims[2],
                                      out_dims[3])
            elif op == "GlobalAveragePool":
                xx = get(nd.inputs[0])
                n, c, h, w = xx.shape
                y = np.zeros(out_dims, np.float32)
                self.L.oracle_global_avg_pool(_fp(np.ascontiguousarray(xx)), n, c, h * w, _fp(y))
            elif op in ("Flatten", "Reshape", "Identity"):
                y = get(nd.inputs[0]).reshape(out_dims).copy()
            elif op == "Gemm":
                al, be, ta, tb = struct.unpack(ennf.GEMM_PARAMS_FMT, nd.params[:12])
                a, b = get(nd.inputs[0]), get(nd.inputs[1])
                c = get(nd.inputs[2]) if len(nd.inputs) > 2 else None
                mm = a.shape[1] if ta else a.shape[0]
                kk = a.shape[0] if ta else a.shape[1]
                nn = b.shape[0] if tb else b.shape[1]
                y = self.gemm(a, b, c, mm, nn, kk, ta, tb, al, be)
            elif op == "Add":
                a, b = get(nd.inputs[0]), get(nd.inputs[1])
                y = np.zeros(out_dims, np.float32)
                self.L.oracle_add(_fp(np.ascontiguousarray(a)), a.size, _fp(np.ascontiguousarray(b)), b.size, _fp(y),
                                  y.size)
            elif op == "Relu":
                a = np.ascontiguousarray(get(nd.inputs[0]))
                y = np.zeros(out_dims, np.float32)
                self.L.oracle_relu(_fp(a), _fp(y), a.size)
            elif op == "MatMul":
                y = self.matmul(get(nd.inputs[0]), get(nd.inputs[1])).reshape(out_dims)
            elif op == "TopK":
                v, ix = self.topk(get(nd.inputs[0]), int(np.asarray(get(nd.inputs[1])).reshape(-1)[0]))
                vals[nd.outputs[1]] = ix.reshape(m.tensors[nd.outputs[1]].dims)
                y = v
            else:
                raise NotImplementedError(f"port oracle: operator {op} ({nd.op_type})")
            vals[nd.outputs[0]] = y.reshape(out_dims)
        return {tid: vals[tid].reshape(-1) for tid in m.outputs}
