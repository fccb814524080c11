"""The slice of the Strata IR a host needs to hand a subgraph to a plugin.

Mirrors crates/ferrite-strata/src/{dtype,shape,graph,attrs}.rs (DType with its
QuantSpec, ShapeClass, Graph/GraphBuilder/Op/Node/Value) and the wire encoder of
crates/ferrite-strata-plugin-api/src/wire/{mod,graph,caps}.rs, byte for byte.
"""
from __future__ import annotations

import re
import struct
from dataclasses import dataclass, field
from typing import Any, Optional

from . import abi

# ---- dtypes (dtype.rs:41-347, raw.rs:154-227) ----------------------------
ELEM = {"f8e5m2": 0, "f8e4m3": 2, "f16": 3, "f32": 4, "f64": 5, "i8": 6, "i16": 7, "i32": 8,
        "i64": 9, "u8": 10, "bool": 11, "f8e8m0": 12, "f4e2m1": 13, "bf16": 14}
ELEM_BYTES = {0: 1, 2: 1, 3: 2, 4: 4, 5: 8, 6: 1, 7: 2, 8: 4, 9: 8, 10: 1, 11: 1, 12: 1, 13: 2, 14: 2}
INT_ELEMS = {6, 7, 8, 9, 10, 11}
QUANT_NONE, QUANT_BLOCK, QUANT_MX = 0, 1, 2


@dataclass(frozen=True)
class DType:
    element: int
    quant_kind: int = QUANT_NONE
    block_size: int = 0
    symmetric: int = 0

    @staticmethod
    def plain(name: str) -> "DType":
        e = ELEM[name]
        if e in INT_ELEMS:
            raise ValueError("a bare integer dtype has no numeric meaning (dtype.rs:306-312)")
        return DType(e)

    @staticmethod
    def quantised(name: str, block_size: int, symmetric: bool = True) -> "DType":
        e = ELEM[name]
        if e not in INT_ELEMS:
            raise ValueError("a quantisation spec on a non-integer element type is a contradiction")
        return DType(e, QUANT_BLOCK, block_size, int(symmetric))

    @staticmethod
    def microscaled(name: str, block_size: int = 32) -> "DType":
        """f8e8m0 or f4e2m1 sharing one E8M0 exponent per block of 32
        (DType::microscaled, dtype.rs)."""
        e = ELEM[name]
        if e not in (ELEM["f8e8m0"], ELEM["f4e2m1"]) or block_size != 32:
            raise ValueError("only f8e8m0 / f4e2m1 with a block of 32 are microscaled")
        return DType(e, QUANT_MX, block_size, 0)

    @property
    def nbytes(self) -> int:
        """Bytes per element as the reference sizes them (f4e2m1: 2)."""
        return ELEM_BYTES[self.element]

    def byte_len(self, elements: int) -> int:
        """Bytes a tensor of `elements` values occupies here: f4e2m1 codes
        are packed two per byte (even index in the low nibble), where the
        reference's ElementType::size_in_bytes reports 2 bytes per element;
        a buffer of the reference's size is accepted (it is larger)."""
        if self.element == ELEM["f4e2m1"]:
            return (elements + 1) // 2
        return elements * ELEM_BYTES[self.element]

    def to_raw(self) -> abi.StrataDType:
        d = abi.StrataDType()
        d.element = self.element
        d.quant.kind = self.quant_kind
        d.quant.block_size = self.block_size
        d.quant.symmetric = self.symmetric
        return d


F32 = DType.plain("f32")
BF16 = DType.plain("bf16")
I32 = DType.quantised("i32", 1)          # token ids and positions
W4G32 = DType.quantised("u8", 32)        # packed int4 codes, group 32 along k
E4M3 = DType.plain("f8e4m3")             # MXFP8 weight codes
E2M1 = DType.microscaled("f4e2m1")       # MXFP4 weight codes, two per byte
E8M0 = DType.microscaled("f8e8m0")       # MX block scales, one per 32 codes along k


def w8pc(k: int) -> DType:
    """int8 codes with one scale per output channel: a block of the whole row."""
    return DType.quantised("i8", k)


# ---- shape classes (shape.rs:225-256) -------------------------------------
SHAPE_SCALAR, SHAPE_EMPTY, SHAPE_OUTER, SHAPE_VECTOR, SHAPE_MATRIX, SHAPE_B3, SHAPE_B4, SHAPE_HIGH = range(8)
MAX_RANK = 8


def shape_class(dims: tuple[int, ...]) -> tuple[int, int]:
    if len(dims) == 0:
        return SHAPE_SCALAR, 0
    if any(d == 0 for d in dims):
        return SHAPE_EMPTY, 0
    if dims[0] == 1:
        return SHAPE_OUTER, 0
    r = len(dims)
    if r == 1:
        return SHAPE_VECTOR, 0
    if r == 2:
        return SHAPE_MATRIX, 0
    if r == 3:
        return SHAPE_B3, 0
    if r == 4:
        return SHAPE_B4, 0
    return SHAPE_HIGH, r


# ---- ops (graph.rs:56-128, raw.rs:296-331) ---------------------------------
OP = {"input": 0, "add": 1, "mul": 2, "matmul": 3, "log": 4, "exp": 5, "softmax": 6,
      "layer_norm": 7, "gelu": 8, "linear": 9, "reshape": 10, "transpose": 11, "expand": 12,
      "slice": 13, "custom": 14}


@dataclass
class Op:
    kind: str
    axis: int = -1
    gamma: int = 0
    beta: int = 0
    eps: float = 1e-5
    weight: int = 0
    bias: Optional[int] = None
    shape: tuple[int, ...] = ()
    permutation: tuple[int, ...] = ()
    start: int = 0
    end: int = 0
    stride: int = 1
    pattern_id: str = ""

    @staticmethod
    def custom(pattern_id: str) -> "Op":
        return Op("custom", pattern_id=pattern_id)

    def pattern(self) -> str:
        """The capability-table id the partitioner asks about (partition.rs:532-584)."""
        if self.kind == "custom":
            return self.pattern_id
        if self.kind in ("slice", "input"):
            return "ref::reshape"
        return "ref::" + self.kind


@dataclass
class Value:
    dtype: DType
    dims: tuple[int, ...]
    producer: Optional[int]
    slot: int
    name: str

    @property
    def elements(self) -> int:
        n = 1
        for d in self.dims:
            n *= d
        return n

    @property
    def nbytes(self) -> int:
        return self.dtype.byte_len(self.elements)


@dataclass
class Node:
    op: Op
    inputs: list[int]
    outputs: list[int]
    attrs: dict[str, Any]
    name: str


@dataclass
class Graph:
    name: str
    values: list[Value] = field(default_factory=list)
    nodes: list[Node] = field(default_factory=list)
    outputs: list[int] = field(default_factory=list)


_KEY = re.compile(r"^[a-z][a-z0-9_]{0,63}$")


class GraphBuilder:
    """graph.rs:617-743: inputs first, then nodes in topological order."""

    def __init__(self, name: str):
        self.g = Graph(name)
        self._names: set[str] = set()

    def _claim(self, name: str) -> None:
        if name in self._names:
            raise ValueError(f"name `{name}` is already used")
        self._names.add(name)

    def input(self, dtype: DType, dims, name: str) -> int:
        dims = tuple(int(d) for d in dims)
        if len(dims) > MAX_RANK:
            raise ValueError("rank too high")
        self._claim(name)
        self.g.values.append(Value(dtype, dims, None, 0, name))
        return len(self.g.values) - 1

    def node(self, op: Op, inputs, outputs, attrs=None, name: str = "") -> list[int]:
        attrs = dict(attrs or {})
        for k in attrs:
            if not _KEY.match(k):
                raise ValueError(f"attribute key `{k}` is not snake_case (attrs.rs:151-178)")
        for i in inputs:
            if not 0 <= i < len(self.g.values):
                raise ValueError(f"unknown value {i}")
        self._claim(name)
        idx = len(self.g.nodes)
        outs = []
        for slot, (dtype, dims) in enumerate(outputs):
            vname = f"{name}#{slot}"
            self._claim(vname)
            self.g.values.append(Value(dtype, tuple(int(d) for d in dims), idx, slot, vname))
            outs.append(len(self.g.values) - 1)
        self.g.nodes.append(Node(op, list(inputs), outs, attrs, name))
        return outs

    def output(self, v: int) -> None:
        if v in self.g.outputs:
            raise ValueError("already an output")
        self.g.outputs.append(v)

    def build(self) -> Graph:
        return self.g


# ---- wire encoding (wire/mod.rs:142-191, wire/graph.rs:101-222) ------------
class _W:
    def __init__(self):
        self.b = bytearray()

    def u8(self, v):
        self.b += struct.pack("<B", v & 0xFF)

    def u32(self, v):
        self.b += struct.pack("<I", v & 0xFFFFFFFF)

    def u64(self, v):
        self.b += struct.pack("<Q", v & 0xFFFFFFFFFFFFFFFF)

    def f32(self, v):
        self.b += struct.pack("<f", v)

    def str(self, s: str):
        raw = s.encode()
        self.u32(len(raw))
        self.b += raw


GRAPH_SCHEMA = 1
SECTION_GRAPH, SECTION_CAPS = 1, 2


def encode_graph(g: Graph) -> bytes:
    w = _W()
    w.u32(GRAPH_SCHEMA)
    w.str(g.name)
    w.u32(len(g.values))
    for v in g.values:
        w.u32(v.dtype.element)
        w.u32(v.dtype.quant_kind)
        w.u32(v.dtype.block_size)
        w.u8(v.dtype.symmetric)
        w.u32(len(v.dims))
        for d in v.dims:
            w.u64(d)
        w.u64(0xFFFFFFFFFFFFFFFF if v.producer is None else (v.producer | (1 << 63)))
        w.u32(v.slot)
        w.str(v.name)
    w.u32(len(g.nodes))
    for n in g.nodes:
        op = n.op
        w.u32(OP[op.kind])
        if op.kind == "softmax":
            w.u64(op.axis)
        elif op.kind == "layer_norm":
            w.u32(op.gamma)
            w.u32(op.beta)
            w.f32(op.eps)
        elif op.kind == "linear":
            w.u32(op.weight)
            if op.bias is None:
                w.u8(0)
            else:
                w.u8(1)
                w.u32(op.bias)
        elif op.kind in ("reshape", "expand"):
            w.u32(len(op.shape))
            for d in op.shape:
                w.u64(d)
        elif op.kind == "transpose":
            w.u32(len(op.permutation))
            for a in op.permutation:
                w.u64(a)
        elif op.kind == "slice":
            w.u64(op.axis)
            w.u64(op.start)
            w.u64(op.end)
            w.u64(op.stride)
        elif op.kind == "custom":
            w.str(op.pattern_id)
        w.u32(len(n.inputs))
        for i in n.inputs:
            w.u32(i)
        w.u32(len(n.outputs))
        for o in n.outputs:
            w.u32(o)
        w.u32(len(n.attrs))
        for k, v in n.attrs.items():
            w.str(k)
            if isinstance(v, bool):
                w.u8(2)
                w.u8(int(v))
            elif isinstance(v, int):
                w.u8(0)
                w.u64(v)
            elif isinstance(v, float):
                w.u8(1)
                w.f32(v)
            elif isinstance(v, str):
                w.u8(3)
                w.str(v)
            else:
                w.u8(4)
                w.u32(len(v))
                for item in v:
                    w.u64(int(item))
        w.str(n.name)
    w.u32(len(g.outputs))
    for o in g.outputs:
        w.u32(o)
    return bytes(w.b)


def frame(sections: list[tuple[int, bytes]]) -> bytes:
    """Blob::finish: header, count, table, then the sections (wire/mod.rs:142-176)."""
    table_bytes = 20 * len(sections)
    base = 4 + table_bytes
    body = bytearray()
    table = _W()
    table.u32(len(sections))
    for kind, data in sections:
        table.u32(kind)
        table.u64(base + len(body))
        table.u64(len(data))
        body += data
    payload = bytes(table.b) + bytes(body)
    head = _W()
    head.u64(abi.MAGIC)
    head.u32(abi.FORMAT_MAJOR)
    head.u32(abi.FORMAT_MINOR)
    head.u64(len(payload))
    return bytes(head.b) + payload


# ---- capability decoding (wire/caps.rs:126-227) ----------------------------
class WireError(ValueError):
    pass


class _R:
    def __init__(self, b: bytes):
        self.b, self.at = b, 0

    def take(self, n):
        if n > len(self.b) - self.at:
            raise WireError(f"truncated: needed {n}, {len(self.b) - self.at} available")
        r = self.b[self.at:self.at + n]
        self.at += n
        return r

    def u8(self):
        return self.take(1)[0]

    def u32(self):
        return struct.unpack("<I", self.take(4))[0]

    def u64(self):
        return struct.unpack("<Q", self.take(8))[0]

    def str(self):
        n = self.u32()
        if n > len(self.b) - self.at:
            raise WireError("length overflow")
        return self.take(n).decode("utf-8")


def parse_sections(blob: bytes) -> dict[int, bytes]:
    """Parsed::parse (wire/mod.rs:241-299): unknown or out-of-range sections are skipped."""
    r = _R(blob)
    if r.u64() != abi.MAGIC:
        raise WireError("bad magic")
    major, _minor, plen = r.u32(), r.u32(), r.u64()
    if major != abi.FORMAT_MAJOR:
        raise WireError("unsupported format")
    payload = blob[abi.WIRE_HEADER_LEN:abi.WIRE_HEADER_LEN + plen]
    if len(payload) < plen:
        raise WireError("truncated payload")
    t = _R(payload)
    out = {}
    for _ in range(t.u32()):
        if len(payload) - t.at < 20:
            break
        kind, off, ln = t.u32(), t.u64(), t.u64()
        if off + ln <= len(payload) and kind in (SECTION_GRAPH, SECTION_CAPS):
            out.setdefault(kind, payload[off:off + ln])
    return out


@dataclass
class PatternSupport:
    pattern_id: str
    dtype: DType
    shape_kind: int
    shape_rank: int
    level: int
    reason: Optional[str]


@dataclass
class CapabilitySet:
    backend_name: str
    patterns: list[PatternSupport]
    compute_units: list[tuple[int, str, str, Optional[int]]]
    max_allocation_bytes: Optional[int]
    max_rank: Optional[int]
    dtype_mask: int
    accepts_unpartitioned: bool


def decode_caps(section: bytes) -> CapabilitySet:
    r = _R(section)
    if r.u32() != 1:
        raise WireError("unsupported caps schema")
    name = r.str()
    pats = []
    for _ in range(r.u32()):
        pid = r.str()
        dt = DType(r.u32(), r.u32(), r.u32(), r.u8())
        kind, rank = r.u32(), r.u8()
        level = r.u32()
        if level > 2:
            raise WireError("unknown support level")
        reason = r.str() if r.u8() else None
        pats.append(PatternSupport(pid, dt, kind, rank, level, reason))
    units = []
    for _ in range(r.u32()):
        idx, uname, kind = r.u32(), r.str(), r.str()
        mem = r.u64() if r.u8() else None
        units.append((idx, uname, kind, mem))
    unset = 0xFFFFFFFFFFFFFFFF
    max_alloc = r.u64()
    r.u64()
    max_rank = r.u32()
    r.u64()
    r.u64()
    mask = r.u32()
    acc = r.u8() != 0
    return CapabilitySet(name, pats, units, None if max_alloc == unset else max_alloc,
                         None if max_rank == 0xFFFFFFFF else max_rank, mask, acc)
