"""ENNF v2 file format: constants, reader, and a graph -> fused ``.ennf`` converter.

The byte layout is SPINN's and must stay identical so that a converted model runs
unchanged on either runtime:

* ``ENNF_Header`` (64 B, ``SPINN/ennf_def.h:70-95``): magic, version, counts, offsets;
  ``reserved[0]`` holds the offset of the dense WeightEntry table
  (``SPINN/onnx2ennf.c:282-291``).
* ``ENNF_WeightEntry`` (16 B, ``ennf_def.h:144-150``), one per tensor id.
* graph meta: ``u16 n_in, u16 in_ids[], u16 n_out, u16 out_ids[]`` (``ennf_def.h:155-160``).
* node table: ``ENNF_NodeBase`` (8 B, ``ennf_def.h:106-119``) + ``u16`` input ids +
  ``u16`` output ids + params (``ennf_op_params.h``).
* ``ENNF_TensorMeta`` (44 B as compiled, ``ennf_def.h:130-139``).
* weight blob, 16-B aligned start, tensors packed back to back (``onnx2ennf.c:432-518``).

:func:`convert` restates the reference converter (``SPINN/onnx2ennf.c:157-529``) and its
fusion passes (``SPINN/graph_opt.c:95-559``) on a :class:`spinn_b200.netdef.Graph`, so
that the benchmark can produce models with no reference code present.  Its output is
checked byte for byte against the reference converter in ``tests/test_ennf_format.py``.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import numpy as np

MAGIC = 0x454E4E46
VERSION = (2, 0)

# ENNF_OpType values (SPINN/ennf_op_types.h:20-300) for the operators this project emits.
OP = {
    "Add": 4, "Div": 23, "Mul": 39, "Sub": 50,
    "Conv": 60,
    "AveragePool": 80, "GlobalAveragePool": 81, "MaxPool": 85,
    "BatchNormalization": 100,
    "Relu": 130, "Sigmoid": 133, "Softmax": 134,
    "Gemm": 160, "MatMul": 161,
    "Concat": 183, "Flatten": 189, "Identity": 193, "Reshape": 197, "Resize": 198,
    "Split": 206, "TopK": 210, "Transpose": 211,
}
OP_NAME = {v: k for k, v in OP.items()}

# fused_act codes carried in ENNF_ConvParams.reserved (SPINN/graph_opt.h:31-36)
ACT_NONE, ACT_RELU, ACT_CLIP, ACT_SILU, ACT_ADD, ACT_ADD_RELU = 0, 1, 2, 3, 4, 5

NODE_FLAG_FUSED = 1          # ENNF_NODE_FLAG_FUSED (ennf_def.h:122)
AUTOPAD = {"NOTSET": 0, "SAME_UPPER": 1, "SAME_LOWER": 2, "VALID": 3}

HEADER_FMT = "<IHHIIIIHHHHIIIII3I"      # 64 bytes
NODEBASE_FMT = "<HBBHBB"                # 8 bytes
META_FMT = "<HBB8IIBB2x"                # 44 bytes
WENTRY_FMT = "<HHIII"                   # 16 bytes
CONV_PARAMS_FMT = "<4H4H8H4HHBB"        # ENNF_ConvParams, 44 bytes
POOL_PARAMS_FMT = "<4H4H8H4HBBBBi"      # ENNF_PoolParams, 48 bytes
GEMM_PARAMS_FMT = "<ffBB2x"             # ENNF_GemmParams, 12 bytes
BN_PARAMS_FMT = "<ffB3x"                # ENNF_BatchNormParams, 12 bytes
assert struct.calcsize(HEADER_FMT) == 64 and struct.calcsize(META_FMT) == 44
assert struct.calcsize(CONV_PARAMS_FMT) == 44 and struct.calcsize(POOL_PARAMS_FMT) == 48


# ============================================================================ reading
@dataclass
class ConvParams:
    kernel_shape: Tuple[int, ...]
    strides: Tuple[int, ...]
    pads: Tuple[int, ...]
    dilations: Tuple[int, ...]
    group: int
    auto_pad: int
    fused_act: int

    @staticmethod
    def unpack(b: bytes) -> "ConvParams":
        v = struct.unpack(CONV_PARAMS_FMT, b[:44])
        return ConvParams(v[0:4], v[4:8], v[8:16], v[16:20], v[20], v[21], v[22])


@dataclass
class EnnfNode:
    op_type: int
    inputs: List[int]
    outputs: List[int]
    params: bytes
    flags: int = 0


@dataclass
class EnnfTensor:
    id: int
    dtype: int
    dims: Tuple[int, ...]
    elem_count: int
    is_weight: int
    ref_count: int


@dataclass
class EnnfModel:
    header: Tuple
    inputs: List[int]
    outputs: List[int]
    nodes: List[EnnfNode]
    tensors: Dict[int, EnnfTensor]
    weights: Dict[int, np.ndarray] = field(default_factory=dict)


def read(data: bytes) -> EnnfModel:
    """Parses a ``.ennf`` image (mirrors ``spinn_load``, ``SPINN/run_time/spinn_runtime.c:21-124``)."""
    h = struct.unpack_from(HEADER_FMT, data, 0)
    if h[0] != MAGIC:
        raise ValueError("not an ENNF file (bad magic)")
    num_nodes, num_tensors = h[3], h[4]
    graph_meta, node_tab, meta_tab, wdata = h[11], h[12], h[13], h[14]
    entry_tab = h[16]
    p = graph_meta
    n_in = struct.unpack_from("<H", data, p)[0]; p += 2
    ins = list(struct.unpack_from(f"<{n_in}H", data, p)); p += 2 * n_in
    n_out = struct.unpack_from("<H", data, p)[0]; p += 2
    outs = list(struct.unpack_from(f"<{n_out}H", data, p))
    nodes = []
    p = node_tab
    for _ in range(num_nodes):
        op, ni, no, ps, fl, _r = struct.unpack_from(NODEBASE_FMT, data, p); p += 8
        ii = list(struct.unpack_from(f"<{ni}H", data, p)); p += 2 * ni
        oo = list(struct.unpack_from(f"<{no}H", data, p)); p += 2 * no
        nodes.append(EnnfNode(op, ii, oo, bytes(data[p:p + ps]), fl)); p += ps
    tensors = {}
    p = meta_tab
    for _ in range(num_tensors):
        v = struct.unpack_from(META_FMT, data, p); p += 44
        t = EnnfTensor(v[0], v[1], tuple(v[3:3 + v[2]]), v[11], v[12], v[13])
        tensors[t.id] = t
    weights = {}
    for tid, t in tensors.items():
        if not t.is_weight:
            continue
        _id, _r, off, size, _r2 = struct.unpack_from(WENTRY_FMT, data, entry_tab + 16 * tid)
        if size:
            dt = np.int64 if t.dtype == 7 else np.float32
            weights[tid] = np.frombuffer(data, dt, size // np.dtype(dt).itemsize, wdata + off).reshape(t.dims)
    return EnnfModel(h, ins, outs, nodes, tensors, weights)


# ============================================================================ converting
_SKIP = 1
_HAS_ACT = 2


class _Fuser:
    """Restatement of the graph_opt passes on a copy of the graph (``SPINN/graph_opt.c``)."""

    def __init__(self, g):
        self.g = g
        self.n = len(g.nodes)
        self.flags = [0] * self.n
        self.act = [0] * self.n
        self.output_names = {name for name, _ in g.outputs}

    def consumers(self, name: str, start: int) -> int:
        # count_consumers, graph_opt.c:52-70: every input slot of every live node from
        # `start`, plus graph outputs.
        c = 0
        for i in range(start, self.n):
            if self.flags[i] & _SKIP:
                continue
            c += sum(1 for x in self.g.nodes[i].inputs if x == name)
        return c + (1 if name in self.output_names else 0)

    def fuse_conv_bn(self) -> int:            # graph_opt.c:95-225
        g, fused = self.g, 0
        for i in range(self.n - 1):
            conv = g.nodes[i]
            if self.flags[i] & _SKIP or conv.op_type != "Conv" or not conv.outputs:
                continue
            out = conv.outputs[0]
            if self.consumers(out, i + 1) != 1:
                continue
            bn, bn_idx = None, 0
            for j in range(i + 1, self.n):
                if self.flags[j] & _SKIP:
                    continue
                nd = g.nodes[j]
                if nd.inputs and nd.inputs[0] == out:
                    if nd.op_type == "BatchNormalization":
                        bn, bn_idx = nd, j
                    break
            if bn is None or len(bn.inputs) < 5:
                continue
            params = [g.initializers.get(x) for x in bn.inputs[1:5]]
            if any(p is None for p in params):
                continue
            scale, bias, mean, var = params
            eps = np.float32(bn.attrs.get("epsilon", 1e-5))
            if len(conv.inputs) < 2 or conv.inputs[1] not in g.initializers:
                continue
            w = g.initializers[conv.inputs[1]]
            oc = w.shape[0] if w.ndim else 0
            if oc <= 0 or scale.size != oc:
                continue
            has_bias = len(conv.inputs) >= 3 and conv.inputs[2] != ""
            cb = g.initializers.get(conv.inputs[2]) if has_bias else None
            factor = (scale / np.sqrt(var + eps)).astype(np.float32)
            w2 = w.reshape(oc, -1)
            w2 *= factor[:, None]                      # in place, float32 (graph_opt.c:183)
            b_old = np.zeros(oc, np.float32)
            if cb is not None:
                nb = min(cb.size, oc)
                b_old[:nb] = cb.reshape(-1)[:nb]
            bias[...] = factor * (b_old - mean) + bias  # graph_opt.c:197, float32
            conv.outputs[0] = bn.outputs[0]
            if not has_bias:
                conv.inputs = conv.inputs[:2] + [bn.inputs[2]]
            else:
                conv.inputs[2] = bn.inputs[2]
            self.flags[bn_idx] = _SKIP
            fused += 1
        return fused

    def _producer_before(self, name: str, i: int) -> bool:
        for k in range(i):
            if name in self.g.nodes[k].outputs:
                return True
        return any(n == name for n, _ in self.g.inputs)

    def fuse_conv_add(self) -> int:           # graph_opt.c:304-421
        g, fused = self.g, 0
        for i in range(self.n - 1):
            conv = g.nodes[i]
            if self.flags[i] & _SKIP or self.act[i] != ACT_NONE:
                continue
            if conv.op_type != "Conv" or not conv.outputs:
                continue
            out = conv.outputs[0]
            if self.consumers(out, i + 1) != 1:
                continue
            add, add_idx = None, 0
            for j in range(i + 1, self.n):
                if self.flags[j] & _SKIP:
                    continue
                nd = g.nodes[j]
                if out in nd.inputs:
                    if nd.op_type == "Add" and len(nd.inputs) == 2:
                        add, add_idx = nd, j
                    break
            if add is None:
                continue
            if add.inputs[0] == out:
                res = add.inputs[1]
            elif add.inputs[1] == out:
                res = add.inputs[0]
            else:
                continue
            if res in g.initializers or not self._producer_before(res, i):
                continue
            relu, relu_idx = None, 0
            aout = add.outputs[0]
            if self.consumers(aout, add_idx + 1) == 1:
                for j in range(add_idx + 1, self.n):
                    if self.flags[j] & _SKIP:
                        continue
                    nd = g.nodes[j]
                    if nd.inputs and nd.inputs[0] == aout:
                        if nd.op_type == "Relu":
                            relu, relu_idx = nd, j
                        break
            if relu is not None:
                conv.outputs[0] = relu.outputs[0]
                self.flags[add_idx] = _SKIP
                self.flags[relu_idx] = _SKIP
                self.act[i] = ACT_ADD_RELU
            else:
                conv.outputs[0] = aout
                self.flags[add_idx] = _SKIP
                self.act[i] = ACT_ADD
            self.flags[i] |= _HAS_ACT
            conv.inputs = conv.inputs + [res]
            fused += 1
        return fused

    def fuse_conv_silu(self) -> int:          # graph_opt.c:431-496
        g, fused = self.g, 0
        for i in range(self.n - 2):
            conv = g.nodes[i]
            if self.flags[i] & _SKIP or self.act[i] != ACT_NONE:
                continue
            if conv.op_type != "Conv" or not conv.outputs:
                continue
            out = conv.outputs[0]
            if self.consumers(out, i + 1) != 2:
                continue
            sig = mul = None
            sig_idx = mul_idx = 0
            for j in range(i + 1, self.n):
                if self.flags[j] & _SKIP:
                    continue
                nd = g.nodes[j]
                if out not in nd.inputs:
                    continue
                if nd.op_type == "Sigmoid" and sig is None:
                    sig, sig_idx = nd, j
                elif nd.op_type == "Mul" and mul is None:
                    mul, mul_idx = nd, j
                else:
                    sig = mul = None
                    break
                if sig is not None and mul is not None:
                    break
            if sig is None or mul is None:
                continue
            sout = sig.outputs[0]
            if self.consumers(sout, sig_idx + 1) != 1:
                continue
            if not (len(mul.inputs) == 2 and sout in mul.inputs):
                continue
            conv.outputs[0] = mul.outputs[0]
            self.flags[sig_idx] = _SKIP
            self.flags[mul_idx] = _SKIP
            self.act[i] = ACT_SILU
            self.flags[i] |= _HAS_ACT
            fused += 1
        return fused

    def fuse_conv_relu(self) -> int:          # graph_opt.c:235-288
        g, fused = self.g, 0
        for i in range(self.n - 1):
            conv = g.nodes[i]
            if self.flags[i] & _SKIP or conv.op_type != "Conv" or not conv.outputs:
                continue
            out = conv.outputs[0]
            if self.consumers(out, i + 1) != 1:
                continue
            relu, relu_idx = None, 0
            for j in range(i + 1, self.n):
                if self.flags[j] & _SKIP:
                    continue
                nd = g.nodes[j]
                if nd.inputs and nd.inputs[0] == out:
                    if nd.op_type == "Relu":
                        relu, relu_idx = nd, j
                    break
            if relu is None:
                continue
            conv.outputs[0] = relu.outputs[0]
            self.act[i] = ACT_RELU                  # overwrites an earlier code, as the reference does
            self.flags[i] |= _HAS_ACT
            self.flags[relu_idx] = _SKIP
            fused += 1
        return fused

    def run(self, disable_add: bool = False, disable_silu: bool = False) -> None:
        # pass order and the ≤10 BN iterations: graph_opt.c:515-559
        for _ in range(10):
            if self.fuse_conv_bn() == 0:
                break
        if not disable_add:
            self.fuse_conv_add()
        if not disable_silu:
            self.fuse_conv_silu()
        self.fuse_conv_relu()


def _ints(v, n, fmt_len):
    out = [0] * fmt_len
    for i, x in enumerate(list(v)[:n]):
        out[i] = int(x) & 0xFFFF
    return out


def _params(node, op_code: int, fused_act: int, pbuf: bytearray) -> bytes:
    """ENNF parameter block of `node`.  `pbuf` is the converter's reused 1024-byte scratch
    (params_buf, SPINN/onnx2ennf.c:307): most extractors clear their struct first, but Split
    writes only `axis` and leaves `num_outputs` as whatever the previous node left there
    (onnx2ennf_ops.c:275-280), which a byte-identical writer has to reproduce."""
    a = node.attrs
    if op_code == OP["Split"]:
        struct.pack_into("<i", pbuf, 0, int(a.get("axis", 0)))
        return bytes(pbuf[:8])
    if op_code == OP["TopK"]:
        # ENNF_TopKParams {i32 axis; u8 largest, sorted, reserved[2]} (ennf_op_params.h:218-224):
        # the extractor (onnx2ennf_ops.c:331-337) leaves `reserved` as the scratch held it
        struct.pack_into("<iBB", pbuf, 0, int(a.get("axis", -1)), int(a.get("largest", 1)) & 0xFF,
                         int(a.get("sorted", 1)) & 0xFF)
        return bytes(pbuf[:8])
    out = _params_fixed(node, op_code, fused_act)
    pbuf[:len(out)] = out
    return out


def _params_fixed(node, op_code: int, fused_act: int) -> bytes:
    a = node.attrs
    if op_code == OP["Conv"]:
        return struct.pack(CONV_PARAMS_FMT, *_ints(a.get("kernel_shape", []), 4, 4),
                           *_ints(a.get("strides", []), 4, 4), *_ints(a.get("pads", []), 8, 8),
                           *_ints(a.get("dilations", []), 4, 4), int(a.get("group", 1)) & 0xFFFF,
                           AUTOPAD.get(a.get("auto_pad", "NOTSET"), 0), fused_act)
    if op_code in (OP["MaxPool"], OP["AveragePool"]):
        return struct.pack(POOL_PARAMS_FMT, *_ints(a.get("kernel_shape", []), 4, 4),
                           *_ints(a.get("strides", []), 4, 4), *_ints(a.get("pads", []), 8, 8),
                           *_ints(a.get("dilations", []), 4, 4),
                           AUTOPAD.get(a.get("auto_pad", "NOTSET"), 0), int(a.get("ceil_mode", 0)),
                           int(a.get("count_include_pad", 0)), int(a.get("storage_order", 0)), 0)
    if op_code == OP["Gemm"]:
        return struct.pack(GEMM_PARAMS_FMT, float(a.get("alpha", 1.0)), float(a.get("beta", 1.0)),
                           int(a.get("transA", 0)), int(a.get("transB", 0)))
    if op_code == OP["BatchNormalization"]:
        return struct.pack(BN_PARAMS_FMT, float(a.get("epsilon", 1e-5)),
                           float(a.get("momentum", 0.9)), int(a.get("training_mode", 0)))
    if op_code in (OP["Flatten"], OP["Concat"]):
        return struct.pack("<i", int(a.get("axis", 1)))
    if op_code == OP["Softmax"]:
        return struct.pack("<i", int(a.get("axis", -1)))
    if op_code == OP["Transpose"]:
        perm = list(a.get("perm", []))
        return struct.pack("<8BB3x", *(perm + [0] * (8 - len(perm)))[:8], len(perm))
    return b""


def convert(graph, disable_add: bool = False, disable_silu: bool = False) -> bytes:
    """Returns the ``.ennf`` bytes that the reference converter writes for ``graph``.

    Restates ``SPINN/onnx2ennf.c:157-529``: tensor ids in first-seen order (initializers,
    inputs, outputs, value_info, then node outputs/inputs, ``:184-246``); reference counts
    taken before fusion; graph_opt passes; skipped nodes dropped; ``fused_act`` stored in
    ``ENNF_ConvParams.reserved`` (``:342-347``).  ``graph`` is not modified.
    """
    g = graph.copy()
    ids: Dict[str, int] = {}

    def tid(name: str) -> int:
        if name not in ids:
            ids[name] = len(ids)
        return ids[name]

    for name in g.initializers:
        tid(name)
    for name, _ in g.inputs:
        tid(name)
    for name, _ in g.outputs:
        tid(name)
    for name in g.value_info:
        tid(name)
    refs: Dict[int, int] = {}
    for n in g.nodes:
        for o in n.outputs:
            tid(o)
        for i in n.inputs:
            k = tid(i)
            refs[k] = refs.get(k, 0) + 1

    fz = _Fuser(g)
    fz.run(disable_add, disable_silu)

    shapes: Dict[str, Tuple[int, ...]] = {}
    shapes.update({n: s for n, s in g.inputs})
    shapes.update({n: s for n, s in g.outputs})
    shapes.update(g.value_info)
    names = sorted(ids, key=ids.get)
    nt = len(names)

    graph_meta = struct.pack("<H", len(g.inputs)) + b"".join(struct.pack("<H", ids[n]) for n, _ in g.inputs)
    graph_meta += struct.pack("<H", len(g.outputs)) + b"".join(struct.pack("<H", ids[n]) for n, _ in g.outputs)

    node_blob = bytearray()
    n_eff = 0
    pbuf = bytearray(1024)
    for i, n in enumerate(g.nodes):
        if fz.flags[i] & _SKIP:
            continue
        n_eff += 1
        code = OP[n.op_type]
        p = _params(n, code, fz.act[i] if code == OP["Conv"] else 0, pbuf)
        flags = NODE_FLAG_FUSED if fz.flags[i] & _HAS_ACT else 0
        node_blob += struct.pack(NODEBASE_FMT, code, len(n.inputs), len(n.outputs), len(p), flags, 0)
        node_blob += b"".join(struct.pack("<H", ids[x]) for x in n.inputs)
        node_blob += b"".join(struct.pack("<H", ids[x]) for x in n.outputs)
        node_blob += p

    meta_blob = bytearray()
    for name in names:
        k = ids[name]
        if name in g.initializers:
            arr = g.initializers[name]
            dims, w, dt = arr.shape, 1, (7 if arr.dtype == np.int64 else 1)
        else:
            dims, w = shapes.get(name, ()), 0
            # map_dtype of the value_info elem_type; UNDEFINED (0) without value_info
            dt = getattr(g, "elem_types", {}).get(name, 1) if name in shapes else 0
        dims = tuple(int(d) for d in dims)[:8]
        elem = int(np.prod(dims)) if dims else 1
        meta_blob += struct.pack(META_FMT, k, dt, len(dims), *(list(dims) + [0] * (8 - len(dims))),
                                 elem & 0xFFFFFFFF, w, refs.get(k, 0) & 0xFF)

    entry_off = 64
    graph_off = entry_off + 16 * nt
    node_off = graph_off + len(graph_meta)
    meta_off = node_off + len(node_blob)
    wdata_off = (meta_off + len(meta_blob) + 15) & ~15
    entries = bytearray()
    wblob = bytearray()
    for name in names:
        k = ids[name]
        if name in g.initializers:
            raw = np.ascontiguousarray(g.initializers[name]).tobytes()
            entries += struct.pack(WENTRY_FMT, k, 0, len(wblob), len(raw), 0)
            wblob += raw
        else:
            entries += struct.pack(WENTRY_FMT, k, 0, 0, 0, 0)
    header = struct.pack(HEADER_FMT, MAGIC, VERSION[0], VERSION[1], n_eff, nt, len(g.initializers),
                         len(wblob), len(g.inputs), len(g.outputs), g.opset, 0,
                         graph_off, node_off, meta_off, wdata_off, 0, entry_off, 0, 0)
    out = bytearray(header) + entries + graph_meta + node_blob + meta_blob
    out += b"\0" * (wdata_off - len(out))
    out += wblob
    return bytes(out)
