"""Minimal ONNX protobuf writer (TEST INFRASTRUCTURE).

Serialises a :class:`spinn_b200.netdef.Graph` into an ONNX ``ModelProto`` so that the
reference converter (``oracle/_ref/onnx2ennf``, built from ``SPINN/onnx2ennf.c``) can turn
it into a ``.ennf`` file.  There is no ``onnx`` package in this image, so the protobuf wire
format is written by hand.  Field numbers are those of the ONNX schema vendored by the
reference (``SPINN/onnx.proto3.pb-c.c`` field descriptor tables): ModelProto
{ir_version=1, graph=7, opset_import=8}, GraphProto {node=1, name=2, initializer=5,
input=11, output=12, value_info=13}, NodeProto {input=1, output=2, name=3, op_type=4,
attribute=5}, AttributeProto {name=1, f=2, i=3, ints=8, type=20}, TensorProto {dims=1,
data_type=2, name=8, raw_data=9}, ValueInfoProto {name=1, type=2},
TypeProto {tensor_type=1}, TypeProto.Tensor {elem_type=1, shape=2},
TensorShapeProto {dim=1}, Dimension {dim_value=1}, OperatorSetIdProto {domain=1, version=2}.
"""
from __future__ import annotations

import struct

import numpy as np

# AttributeProto.AttributeType
_ATTR_FLOAT, _ATTR_INT, _ATTR_STRING, _ATTR_INTS = 1, 2, 3, 7
_FLOAT32 = 1
_INT64 = 7


def _varint(v: int) -> bytes:
    if v < 0:
        v += 1 << 64
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(field: int, wire: int) -> bytes:
    return _varint((field << 3) | wire)


def _f_varint(field: int, v: int) -> bytes:
    return _key(field, 0) + _varint(int(v))


def _f_bytes(field: int, data: bytes) -> bytes:
    return _key(field, 2) + _varint(len(data)) + data


def _f_str(field: int, s: str) -> bytes:
    return _f_bytes(field, s.encode())


def _f_float(field: int, v: float) -> bytes:
    return _key(field, 5) + struct.pack("<f", float(v))


def _f_packed_varints(field: int, vals) -> bytes:
    return _f_bytes(field, b"".join(_varint(int(v)) for v in vals))


def _attribute(name: str, value) -> bytes:
    msg = _f_str(1, name)
    if isinstance(value, float):
        msg += _f_float(2, value) + _f_varint(20, _ATTR_FLOAT)
    elif isinstance(value, (int, np.integer)):
        msg += _f_varint(3, int(value)) + _f_varint(20, _ATTR_INT)
    elif isinstance(value, str):
        msg += _f_bytes(4, value.encode()) + _f_varint(20, _ATTR_STRING)
    elif isinstance(value, (list, tuple)):
        msg += _f_packed_varints(8, value) + _f_varint(20, _ATTR_INTS)
    else:
        raise TypeError(f"attribute {name}: unsupported {type(value)}")
    return msg


def _tensor(name: str, arr: np.ndarray) -> bytes:
    is_int = np.asarray(arr).dtype.kind in "iu"
    arr = np.ascontiguousarray(arr, dtype=np.int64 if is_int else np.float32)
    msg = _f_packed_varints(1, arr.shape) if arr.ndim else b""
    msg += _f_varint(2, _INT64 if is_int else _FLOAT32) + _f_str(8, name) + _f_bytes(9, arr.tobytes())
    return msg


def _value_info(name: str, shape, elem_type: int = _FLOAT32) -> bytes:
    dims = b"".join(_f_bytes(1, _f_varint(1, d)) for d in shape)
    tensor_type = _f_varint(1, elem_type) + _f_bytes(2, dims)
    return _f_str(1, name) + _f_bytes(2, _f_bytes(1, tensor_type))


def _node(n) -> bytes:
    msg = b"".join(_f_str(1, i) for i in n.inputs)
    msg += b"".join(_f_str(2, o) for o in n.outputs)
    msg += _f_str(3, n.name or n.op_type) + _f_str(4, n.op_type)
    for k, v in n.attrs.items():
        msg += _f_bytes(5, _attribute(k, v))
    return msg


def graph_to_onnx(g) -> bytes:
    """Returns the serialised ModelProto for graph ``g``."""
    gm = b"".join(_f_bytes(1, _node(n)) for n in g.nodes)
    gm += _f_str(2, g.name)
    gm += b"".join(_f_bytes(5, _tensor(k, v)) for k, v in g.initializers.items())
    et = getattr(g, "elem_types", {})
    gm += b"".join(_f_bytes(11, _value_info(n, s, et.get(n, _FLOAT32))) for n, s in g.inputs)
    gm += b"".join(_f_bytes(12, _value_info(n, s, et.get(n, _FLOAT32))) for n, s in g.outputs)
    gm += b"".join(_f_bytes(13, _value_info(n, s, et.get(n, _FLOAT32))) for n, s in g.value_info.items())
    opset = _f_str(1, "") + _f_varint(2, g.opset)
    return _f_varint(1, 8) + _f_str(2, "spinn_b200.netdef") + _f_bytes(7, gm) + _f_bytes(8, opset)
