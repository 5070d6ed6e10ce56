"""A minimal ONNX ModelProto writer (protobuf wire format, no onnx package).

Writes the subset of onnx.proto3 that nnr's loader reads
(format/onnx/onnx_pb.cpp): ModelProto{ir_version, opset_import, graph},
GraphProto{node, name, initializer, input, output}, NodeProto{input, output,
name, op_type, attribute}, AttributeProto{name, type, f, i, s, floats, ints},
TensorProto{dims, data_type, name, raw_data} and ValueInfoProto with a tensor
type and fixed dims. Used to hand seeded models (the BASELINE configs) to
nnr's own loader: context_t::load(buf, len) (nnr.cpp:771).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field
from typing import Dict, List, Sequence

import numpy as np

# TensorProto.DataType
FLOAT, UINT8, INT8, INT32, INT64, FLOAT16, BFLOAT16 = 1, 2, 3, 6, 7, 10, 16
_NP = {np.dtype(np.float32): FLOAT, np.dtype(np.uint8): UINT8, np.dtype(np.int8): INT8,
       np.dtype(np.int32): INT32, np.dtype(np.int64): INT64, np.dtype(np.float16): FLOAT16}
# AttributeProto.AttributeType
A_FLOAT, A_INT, A_STRING, A_FLOATS, A_INTS = 1, 2, 3, 6, 7


def _varint(v: int) -> bytes:
    v &= (1 << 64) - 1
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(fn: int, wt: int) -> bytes:
    return _varint((fn << 3) | wt)


def _vint(fn: int, v: int) -> bytes:
    return _key(fn, 0) + _varint(int(v))


def _bytes(fn: int, b: bytes) -> bytes:
    return _key(fn, 2) + _varint(len(b)) + b


def _str(fn: int, s: str) -> bytes:
    return _bytes(fn, s.encode())


def _f32(fn: int, v: float) -> bytes:
    return _key(fn, 5) + struct.pack("<f", float(v))


def tensor(name: str, arr: np.ndarray, data_type: int = 0) -> bytes:
    """data_type overrides the element type (BFLOAT16 for uint16 bit patterns)."""
    arr = np.ascontiguousarray(arr)
    dims = b"".join(_varint(int(d)) for d in arr.shape)
    out = _bytes(1, dims) if arr.ndim else b""
    return out + _vint(2, data_type or _NP[arr.dtype]) + _str(8, name) + _bytes(9, arr.tobytes())


def value_info(name: str, elem_type: int, shape: Sequence[int]) -> bytes:
    dims = b"".join(_bytes(1, _vint(1, d)) for d in shape)
    ttype = _vint(1, elem_type) + _bytes(2, dims)
    return _str(1, name) + _bytes(2, _bytes(1, ttype))


def attribute(name: str, v) -> bytes:
    if isinstance(v, float):
        return _str(1, name) + _vint(20, A_FLOAT) + _f32(2, v)
    if isinstance(v, (bool, int, np.integer)):
        return _str(1, name) + _vint(20, A_INT) + _vint(3, int(v))
    if isinstance(v, str):
        return _str(1, name) + _vint(20, A_STRING) + _bytes(4, v.encode())
    v = list(v)
    if all(isinstance(x, (int, np.integer)) for x in v):
        return _str(1, name) + _vint(20, A_INTS) + _bytes(8, b"".join(_varint(int(x)) for x in v))
    return _str(1, name) + _vint(20, A_FLOATS) + _bytes(7, b"".join(struct.pack("<f", float(x)) for x in v))


@dataclass
class Graph:
    """Nodes, initializers and typed graph inputs/outputs, in the order added."""
    name: str = "g"
    nodes: List[bytes] = field(default_factory=list)
    inits: List[bytes] = field(default_factory=list)
    inputs: List[bytes] = field(default_factory=list)
    outputs: List[bytes] = field(default_factory=list)
    _n: int = 0
    _consts: Dict[tuple, str] = field(default_factory=dict)

    def node(self, op: str, ins: Sequence[str], outs: Sequence[str], **attrs) -> str:
        self._n += 1
        b = b"".join(_str(1, i) for i in ins) + b"".join(_str(2, o) for o in outs)
        b += _str(3, f"{op}_{self._n}") + _str(4, op)
        for k, v in attrs.items():
            b += _bytes(5, attribute(k, v))
        self.nodes.append(b)
        return outs[0]

    def init(self, name: str, arr: np.ndarray, data_type: int = 0) -> str:
        self.inits.append(tensor(name, arr, data_type))
        return name

    def scalar(self, arr) -> str:
        """A scalar initializer, shared between nodes that use the same value."""
        arr = np.asarray(arr)
        key = (arr.dtype.str, arr.tobytes())
        if key not in self._consts:
            self._consts[key] = self.init(f"c{len(self._consts)}", arr)
        return self._consts[key]

    def input(self, name: str, elem_type: int, shape: Sequence[int]) -> str:
        self.inputs.append(value_info(name, elem_type, shape))
        return name

    def output(self, name: str, elem_type: int, shape: Sequence[int]) -> str:
        self.outputs.append(value_info(name, elem_type, shape))
        return name

    def model(self, opset: int = 13) -> bytes:
        g = b"".join(_bytes(1, n) for n in self.nodes) + _str(2, self.name)
        g += b"".join(_bytes(5, t) for t in self.inits)
        g += b"".join(_bytes(11, v) for v in self.inputs) + b"".join(_bytes(12, v) for v in self.outputs)
        return _vint(1, 8) + _bytes(8, _str(1, "") + _vint(2, opset)) + _str(2, "nnr_b200") + _bytes(7, g)
