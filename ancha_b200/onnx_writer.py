"""Minimal ONNX (opset 13) model writer for synthetic classic-MDX graphs and tests.

Encodes the protobuf wire format of the ModelProto subset the classic MDX executor reads
(crates/ancha-models/src/mdx.rs:161-472): opset imports, one graph with nodes (inputs,
outputs, name, op_type, INT / INTS / FLOAT attributes), FLOAT initializers (raw little-endian
data) and named inputs / outputs with optional NCHW shapes. Field numbers are those of the
public onnx.proto schema. No onnx package is needed.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np

FLOAT = 1  # TensorProto.DataType.FLOAT
ATTR_FLOAT, ATTR_INT, ATTR_INTS = 1, 2, 7  # AttributeProto.AttributeType


def _varint(v: int) -> bytes:
    v &= (1 << 64) - 1  # negative int64 as ten-byte two's complement
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(field_no: int, wire: int) -> bytes:
    return _varint((field_no << 3) | wire)


def _len(field_no: int, payload: bytes) -> bytes:
    return _key(field_no, 2) + _varint(len(payload)) + payload


def _str(field_no: int, s: str) -> bytes:
    return _len(field_no, s.encode())


def _int(field_no: int, v: int) -> bytes:
    return _key(field_no, 0) + _varint(v)


@dataclass
class Attr:
    name: str
    ints: Optional[Sequence[int]] = None
    i: Optional[int] = None
    f: Optional[float] = None
    packed: bool = True  # onnx.proto (proto2) writers emit INTS unpacked; both forms are valid

    def encode(self) -> bytes:
        out = _str(1, self.name)
        if self.ints is not None:
            if self.packed:
                out += _int(20, ATTR_INTS) + _len(8, b"".join(_varint(v) for v in self.ints))
            else:
                out += _int(20, ATTR_INTS) + b"".join(_int(8, v) for v in self.ints)
        elif self.i is not None:
            out += _int(20, ATTR_INT) + _int(3, self.i)
        elif self.f is not None:
            out += _int(20, ATTR_FLOAT) + _key(2, 5) + struct.pack("<f", self.f)
        return out


@dataclass
class Node:
    op_type: str
    inputs: Sequence[str]
    output: str
    name: str = ""
    attrs: Sequence[Attr] = field(default_factory=list)
    domain: str = ""

    def encode(self) -> bytes:
        out = b"".join(_str(1, s) for s in self.inputs) + _str(2, self.output)
        if self.name:
            out += _str(3, self.name)
        out += _str(4, self.op_type)
        out += b"".join(_len(5, a.encode()) for a in self.attrs)
        if self.domain:
            out += _str(7, self.domain)
        return out


def tensor(name: str, array, float_data: bool = False) -> bytes:
    """TensorProto of a FLOAT array: dims, data_type, name and raw_data (or packed float_data)."""
    a = np.ascontiguousarray(array, dtype="<f4")
    out = b"".join(_int(1, d) for d in a.shape) + _int(2, FLOAT) + _str(8, name)
    return out + (_len(4, a.tobytes()) if float_data else _len(9, a.tobytes()))


def value_info(name: str, shape: Optional[Sequence[int]] = None) -> bytes:
    out = _str(1, name)
    if shape is not None:
        dims = b"".join(_len(1, _int(1, d)) for d in shape)
        tensor_type = _int(1, FLOAT) + _len(2, dims)
        out += _len(2, _len(1, tensor_type))
    return out


def model(nodes: Sequence[Node], initializers: dict, inputs=("x",), outputs=("out",),
          input_shape=None, output_shape=None, opset: int = 13, ir_version: int = 7,
          float_data: bool = False, raw_tensors: Sequence[bytes] = ()) -> bytes:
    """ModelProto bytes: one graph over `nodes` with FLOAT `initializers` (name → array) and
    `raw_tensors`, TensorProto payloads encoded by the caller (for malformed-input tests)."""
    g = b"".join(_len(1, n.encode()) for n in nodes) + _str(2, "graph")
    g += b"".join(_len(5, tensor(k, v, float_data)) for k, v in initializers.items())
    g += b"".join(_len(5, t) for t in raw_tensors)
    g += b"".join(_len(11, value_info(n, input_shape)) for n in inputs)
    g += b"".join(_len(12, value_info(n, output_shape)) for n in outputs)
    opset_id = _str(1, "") + _int(2, opset)
    return _int(1, ir_version) + _len(8, opset_id) + _len(7, g)
