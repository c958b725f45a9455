"""Minimal ONNX ModelProto reader and writer (protobuf wire format, no ``onnx`` package).

The ``onnx`` and ``onnxruntime`` packages are not installable on the build host, so the
model files this project generates (the BASELINE conv-chain configs and the engine test
fixtures) and the shipped ArtCNN models are written and read here directly at the wire
level. Only the fields the conv-chain path consumes are modelled; unknown fields are
skipped on read, exactly as a protobuf parser would.

Field numbers follow the public ``onnx.proto`` schema (ModelProto, GraphProto,
NodeProto, AttributeProto, TensorProto, ValueInfoProto, TypeProto). The engine's own
C++ decoder (``csrc/onnx_wire.cc``) reads the same subset.

Reference call sites this mirrors: the fixture writer ``tests/correctness/harness/
modelgen.py:57-130`` (helper.make_node / numpy_helper.from_array / the typed-half
``int32_data`` initializer at :97-107) and the reader side of
``src/vapoursynth/hip_engine.cc:51-112`` (initializer materialisation).
"""

from __future__ import annotations

import struct
from dataclasses import dataclass, field
from typing import Iterable

import numpy as np

# TensorProto.DataType values (onnx.proto).
FLOAT = 1
UINT8 = 2
INT8 = 3
UINT16 = 4
INT16 = 5
INT32 = 6
INT64 = 7
STRING = 8
BOOL = 9
FLOAT16 = 10
DOUBLE = 11
UINT32 = 12
UINT64 = 13
BFLOAT16 = 16

_NP_OF = {
    FLOAT: np.float32,
    FLOAT16: np.float16,
    DOUBLE: np.float64,
    INT64: np.int64,
    INT32: np.int32,
    INT16: np.int16,
    INT8: np.int8,
    UINT8: np.uint8,
    UINT16: np.uint16,
    UINT32: np.uint32,
    UINT64: np.uint64,
    BOOL: np.bool_,
}
_ONNX_OF = {np.dtype(v): k for k, v in _NP_OF.items()}

# AttributeProto.AttributeType values.
ATTR_FLOAT = 1
ATTR_INT = 2
ATTR_STRING = 3
ATTR_TENSOR = 4
ATTR_FLOATS = 6
ATTR_INTS = 7


# ---------------------------------------------------------------------------
# Wire-format primitives
# ---------------------------------------------------------------------------

def _varint(v: int) -> bytes:
    if v < 0:
        v &= (1 << 64) - 1  # two's-complement int64, as protobuf encodes negative ints
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(fnum: int, wtype: int) -> bytes:
    return _varint((fnum << 3) | wtype)


def _f_varint(fnum: int, v: int) -> bytes:
    return _key(fnum, 0) + _varint(int(v))


def _f_bytes(fnum: int, b: bytes) -> bytes:
    return _key(fnum, 2) + _varint(len(b)) + b


def _f_str(fnum: int, s: str) -> bytes:
    return _f_bytes(fnum, s.encode())


def _f_float(fnum: int, v: float) -> bytes:
    return _key(fnum, 5) + struct.pack("<f", v)


def _read_varint(buf: bytes, pos: int) -> tuple[int, int]:
    result = 0
    shift = 0
    while True:
        if pos >= len(buf):
            raise ValueError("truncated varint")
        b = buf[pos]
        pos += 1
        result |= (b & 0x7F) << shift
        if not b & 0x80:
            return result, pos
        shift += 7
        if shift > 63:
            raise ValueError("varint too long")


def _fields(buf: bytes):
    """Yield (field_number, wire_type, value) over one message's bytes."""
    pos = 0
    n = len(buf)
    while pos < n:
        key, pos = _read_varint(buf, pos)
        fnum, wt = key >> 3, key & 7
        if wt == 0:
            v, pos = _read_varint(buf, pos)
        elif wt == 1:
            v = buf[pos:pos + 8]
            pos += 8
        elif wt == 2:
            ln, pos = _read_varint(buf, pos)
            v = buf[pos:pos + ln]
            if len(v) != ln:
                raise ValueError("truncated length-delimited field")
            pos += ln
        elif wt == 5:
            v = buf[pos:pos + 4]
            pos += 4
        else:
            raise ValueError(f"unsupported wire type {wt}")
        yield fnum, wt, v


def _signed64(v: int) -> int:
    return v - (1 << 64) if v >= (1 << 63) else v


def _signed32(v: int) -> int:
    v &= (1 << 64) - 1
    v = _signed64(v)
    return v


def _packed_varints(wt: int, v) -> list[int]:
    if wt == 0:
        return [v]
    vals = []
    pos = 0
    while pos < len(v):
        x, pos = _read_varint(v, pos)
        vals.append(x)
    return vals


# ---------------------------------------------------------------------------
# Data model
# ---------------------------------------------------------------------------

@dataclass
class Tensor:
    name: str
    data_type: int
    dims: list[int]
    raw_data: bytes | None = None
    float_data: list[float] = field(default_factory=list)
    int32_data: list[int] = field(default_factory=list)
    int64_data: list[int] = field(default_factory=list)
    double_data: list[float] = field(default_factory=list)
    external: bool = False

    def to_numpy(self) -> np.ndarray:
        """Decode the stored values with the declared dtype preserved.

        FLOAT16 values in ``int32_data`` are 16-bit bit patterns (one slot per
        element), not numeric integers (``hip_engine.cc:88-103``)."""
        if self.external:
            raise ValueError(f"initializer '{self.name}' uses external data")
        dt = _NP_OF.get(self.data_type)
        if dt is None:
            raise ValueError(f"unsupported dtype {self.data_type}")
        shape = tuple(self.dims)
        if self.raw_data is not None and len(self.raw_data) > 0:
            return np.frombuffer(self.raw_data, dtype=dt).reshape(shape).copy()
        if self.float_data:
            return np.asarray(self.float_data, dtype=np.float32).reshape(shape)
        if self.double_data:
            return np.asarray(self.double_data, dtype=np.float64).reshape(shape)
        if self.int32_data:
            arr = np.asarray(self.int32_data, dtype=np.int64) & 0xFFFFFFFF
            if self.data_type in (FLOAT16, BFLOAT16, UINT16, INT16):
                return arr.astype(np.uint16).view(dt if dt != np.int16 else np.int16).reshape(shape)
            return arr.astype(np.uint32).astype(np.int64).astype(dt).reshape(shape)
        if self.int64_data:
            return np.asarray(self.int64_data, dtype=np.int64).astype(dt).reshape(shape)
        return np.zeros(shape, dtype=dt)


@dataclass
class Attribute:
    name: str
    type: int
    f: float = 0.0
    i: int = 0
    s: bytes = b""
    floats: list[float] = field(default_factory=list)
    ints: list[int] = field(default_factory=list)
    t: Tensor | None = None


@dataclass
class Node:
    op_type: str
    inputs: list[str]
    outputs: list[str]
    attrs: dict[str, Attribute] = field(default_factory=dict)
    name: str = ""
    domain: str = ""

    def attr(self, name: str, default=None):
        a = self.attrs.get(name)
        if a is None:
            return default
        if a.type == ATTR_FLOAT:
            return a.f
        if a.type == ATTR_INT:
            return a.i
        if a.type == ATTR_STRING:
            return a.s.decode()
        if a.type == ATTR_INTS:
            return list(a.ints)
        if a.type == ATTR_FLOATS:
            return list(a.floats)
        if a.type == ATTR_TENSOR:
            return a.t
        return default


@dataclass
class ValueInfo:
    name: str
    elem_type: int
    shape: list  # ints or str (dim_param) or None


@dataclass
class Graph:
    nodes: list[Node]
    inputs: list[ValueInfo]
    outputs: list[ValueInfo]
    initializers: list[Tensor]
    name: str = "graph"


@dataclass
class Model:
    graph: Graph
    opset: int = 17
    ir_version: int = 8
    producer: str = "arthip_b200"


# ---------------------------------------------------------------------------
# Writer
# ---------------------------------------------------------------------------

def _enc_tensor(t: Tensor) -> bytes:
    out = bytearray()
    for d in t.dims:
        out += _f_varint(1, d)
    out += _f_varint(2, t.data_type)
    if t.float_data:
        out += _f_bytes(4, struct.pack(f"<{len(t.float_data)}f", *t.float_data))
    if t.int32_data:
        out += _f_bytes(5, b"".join(_varint(v) for v in t.int32_data))
    if t.int64_data:
        out += _f_bytes(7, b"".join(_varint(v) for v in t.int64_data))
    out += _f_str(8, t.name)
    if t.raw_data is not None:
        out += _f_bytes(9, t.raw_data)
    if t.double_data:
        out += _f_bytes(10, struct.pack(f"<{len(t.double_data)}d", *t.double_data))
    if t.external:
        out += _f_bytes(13, _f_str(1, "location") + _f_str(2, f"{t.name}.bin"))
        out += _f_varint(14, 1)
    return bytes(out)


def _enc_attr(a: Attribute) -> bytes:
    out = bytearray(_f_str(1, a.name))
    out += _f_varint(20, a.type)
    if a.type == ATTR_FLOAT:
        out += _f_float(2, a.f)
    elif a.type == ATTR_INT:
        out += _f_varint(3, a.i)
    elif a.type == ATTR_STRING:
        out += _f_bytes(4, a.s)
    elif a.type == ATTR_TENSOR:
        out += _f_bytes(5, _enc_tensor(a.t))
    elif a.type == ATTR_FLOATS:
        for v in a.floats:
            out += _f_float(7, v)
    elif a.type == ATTR_INTS:
        for v in a.ints:
            out += _f_varint(8, v)
    return bytes(out)


def _enc_node(n: Node) -> bytes:
    out = bytearray()
    for i in n.inputs:
        out += _f_str(1, i)
    for o in n.outputs:
        out += _f_str(2, o)
    if n.name:
        out += _f_str(3, n.name)
    out += _f_str(4, n.op_type)
    for a in n.attrs.values():
        out += _f_bytes(5, _enc_attr(a))
    if n.domain:
        out += _f_str(7, n.domain)
    return bytes(out)


def _enc_value_info(v: ValueInfo) -> bytes:
    shape = bytearray()
    for d in v.shape:
        if isinstance(d, int):
            shape += _f_bytes(1, _f_varint(1, d))
        elif isinstance(d, str):
            shape += _f_bytes(1, _f_str(2, d))
        else:
            shape += _f_bytes(1, b"")
    tensor_type = _f_varint(1, v.elem_type) + _f_bytes(2, bytes(shape))
    type_proto = _f_bytes(1, tensor_type)
    return _f_str(1, v.name) + _f_bytes(2, type_proto)


def encode_model(m: Model) -> bytes:
    g = m.graph
    gb = bytearray()
    for n in g.nodes:
        gb += _f_bytes(1, _enc_node(n))
    gb += _f_str(2, g.name)
    for t in g.initializers:
        gb += _f_bytes(5, _enc_tensor(t))
    for v in g.inputs:
        gb += _f_bytes(11, _enc_value_info(v))
    for v in g.outputs:
        gb += _f_bytes(12, _enc_value_info(v))
    out = bytearray(_f_varint(1, m.ir_version))
    out += _f_str(2, m.producer)
    out += _f_bytes(7, bytes(gb))
    out += _f_bytes(8, _f_str(1, "") + _f_varint(2, m.opset))
    return bytes(out)


def save_model(m: Model, path) -> None:
    with open(path, "wb") as f:
        f.write(encode_model(m))


# Construction helpers (the shape of onnx.helper's API, kept deliberately small).

def make_attr(name: str, value) -> Attribute:
    if isinstance(value, float):
        return Attribute(name, ATTR_FLOAT, f=value)
    if isinstance(value, bool) or isinstance(value, int):
        return Attribute(name, ATTR_INT, i=int(value))
    if isinstance(value, str):
        return Attribute(name, ATTR_STRING, s=value.encode())
    if isinstance(value, (list, tuple)):
        if all(isinstance(v, int) for v in value):
            return Attribute(name, ATTR_INTS, ints=[int(v) for v in value])
        return Attribute(name, ATTR_FLOATS, floats=[float(v) for v in value])
    if isinstance(value, Tensor):
        return Attribute(name, ATTR_TENSOR, t=value)
    raise TypeError(f"unsupported attribute value for {name}: {value!r}")


def make_node(op_type: str, inputs: Iterable[str], outputs: Iterable[str], **attrs) -> Node:
    return Node(op_type, list(inputs), list(outputs), {k: make_attr(k, v) for k, v in attrs.items()})


def tensor_from_array(name: str, array: np.ndarray, *, typed_half: bool = False,
                      external: bool = False) -> Tensor:
    """Initializer from an array. ``typed_half`` stores FLOAT16 bit patterns in
    ``int32_data`` (one slot per element) instead of ``raw_data``."""
    a = np.ascontiguousarray(array)
    dt = _ONNX_OF[a.dtype]
    t = Tensor(name=name, data_type=dt, dims=[int(d) for d in a.shape], external=external)
    if typed_half:
        assert dt == FLOAT16
        t.int32_data = [int(v) for v in a.view(np.uint16).ravel()]
    elif not external:
        t.raw_data = a.tobytes()
    return t


def value_info(name: str, elem_type: int, shape) -> ValueInfo:
    return ValueInfo(name, elem_type, list(shape))


# ---------------------------------------------------------------------------
# Reader
# ---------------------------------------------------------------------------

def _dec_tensor(buf: bytes) -> Tensor:
    t = Tensor(name="", data_type=0, dims=[])
    for fnum, wt, v in _fields(buf):
        if fnum == 1:
            t.dims.extend(_signed64(x) for x in _packed_varints(wt, v))
        elif fnum == 2:
            t.data_type = v
        elif fnum == 4:
            if wt == 5:
                t.float_data.append(struct.unpack("<f", v)[0])
            else:
                t.float_data.extend(struct.unpack(f"<{len(v) // 4}f", v))
        elif fnum == 5:
            t.int32_data.extend(_signed32(x) for x in _packed_varints(wt, v))
        elif fnum == 7:
            t.int64_data.extend(_signed64(x) for x in _packed_varints(wt, v))
        elif fnum == 8:
            t.name = v.decode()
        elif fnum == 9:
            t.raw_data = bytes(v)
        elif fnum == 10:
            if wt == 1:
                t.double_data.append(struct.unpack("<d", v)[0])
            else:
                t.double_data.extend(struct.unpack(f"<{len(v) // 8}d", v))
        elif fnum == 14:
            t.external = (v == 1)
    return t


def _dec_attr(buf: bytes) -> Attribute:
    a = Attribute(name="", type=0)
    for fnum, wt, v in _fields(buf):
        if fnum == 1:
            a.name = v.decode()
        elif fnum == 20:
            a.type = v
        elif fnum == 2:
            a.f = struct.unpack("<f", v)[0]
        elif fnum == 3:
            a.i = _signed64(v)
        elif fnum == 4:
            a.s = bytes(v)
        elif fnum == 5:
            a.t = _dec_tensor(v)
        elif fnum == 7:
            if wt == 5:
                a.floats.append(struct.unpack("<f", v)[0])
            else:
                a.floats.extend(struct.unpack(f"<{len(v) // 4}f", v))
        elif fnum == 8:
            a.ints.extend(_signed64(x) for x in _packed_varints(wt, v))
    if a.type == 0:  # proto files that omit the type tag: infer it
        if a.ints:
            a.type = ATTR_INTS
        elif a.floats:
            a.type = ATTR_FLOATS
        elif a.s:
            a.type = ATTR_STRING
        elif a.t is not None:
            a.type = ATTR_TENSOR
    return a


def _dec_node(buf: bytes) -> Node:
    n = Node(op_type="", inputs=[], outputs=[])
    for fnum, wt, v in _fields(buf):
        if fnum == 1:
            n.inputs.append(v.decode())
        elif fnum == 2:
            n.outputs.append(v.decode())
        elif fnum == 3:
            n.name = v.decode()
        elif fnum == 4:
            n.op_type = v.decode()
        elif fnum == 5:
            a = _dec_attr(v)
            n.attrs[a.name] = a
        elif fnum == 7:
            n.domain = v.decode()
    return n


def _dec_value_info(buf: bytes) -> ValueInfo:
    vi = ValueInfo(name="", elem_type=0, shape=[])
    for fnum, wt, v in _fields(buf):
        if fnum == 1:
            vi.name = v.decode()
        elif fnum == 2:
            for f2, _, v2 in _fields(v):
                if f2 != 1:
                    continue
                for f3, _, v3 in _fields(v2):
                    if f3 == 1:
                        vi.elem_type = v3
                    elif f3 == 2:
                        for f4, _, v4 in _fields(v3):
                            if f4 != 1:
                                continue
                            d = None
                            for f5, _, v5 in _fields(v4):
                                if f5 == 1:
                                    d = _signed64(v5)
                                elif f5 == 2:
                                    d = v5.decode()
                            vi.shape.append(d)
    return vi


def decode_model(buf: bytes) -> Model:
    graph_bytes = None
    opset = 0
    ir = 0
    producer = ""
    for fnum, wt, v in _fields(buf):
        if fnum == 1:
            ir = v
        elif fnum == 2:
            producer = v.decode(errors="replace")
        elif fnum == 7:
            graph_bytes = v
        elif fnum == 8:
            dom, ver = "", 0
            for f2, _, v2 in _fields(v):
                if f2 == 1:
                    dom = v2.decode()
                elif f2 == 2:
                    ver = v2
            if dom in ("", "ai.onnx"):
                opset = ver
    if graph_bytes is None:
        raise ValueError("model has no graph")
    g = Graph(nodes=[], inputs=[], outputs=[], initializers=[])
    for fnum, wt, v in _fields(graph_bytes):
        if fnum == 1:
            g.nodes.append(_dec_node(v))
        elif fnum == 2:
            g.name = v.decode()
        elif fnum == 5:
            g.initializers.append(_dec_tensor(v))
        elif fnum == 11:
            g.inputs.append(_dec_value_info(v))
        elif fnum == 12:
            g.outputs.append(_dec_value_info(v))
    # Graph inputs that are also initializers (older exporters) are not activations.
    init_names = {t.name for t in g.initializers}
    g.inputs = [vi for vi in g.inputs if vi.name not in init_names] or g.inputs
    return Model(graph=g, opset=opset, ir_version=ir, producer=producer)


def load_model(path) -> Model:
    with open(path, "rb") as f:
        return decode_model(f.read())
