"""Programs: a model's step as dataflow (src/FuryKernel/Program/Graph.hs).

Straight-line dataflow over row values: sources (activations, row integers,
weights, tables of weights, KV caches), nodes of a small vocabulary of
operations, and outputs. This restates the reference's types for the host
side of the CUDA target; two additions serve the f32 Llama path the target
runs: the SiLU-gate (`SiluMul`, beside `GeluMul`) and f32 KV caches
(`CACHE_F32`, beside bf16 and f16).
"""

from __future__ import annotations

import struct
from dataclasses import dataclass, field
from typing import Optional


@dataclass(frozen=True)
class Shape:
    """A row's elements: `width` of them in segments of `segment` (Graph.hs:88-100)."""

    width: int
    segment: int

    def segments(self) -> int:
        return 0 if self.segment == 0 else self.width // self.segment


def whole_row(n: int) -> Shape:
    return Shape(n, n)


# ---- sources ---------------------------------------------------------------


@dataclass(frozen=True)
class SInput:
    shape: Shape
    type: str


@dataclass(frozen=True)
class SRowInts:
    count: int
    bound: int


@dataclass(frozen=True)
class SWeight:
    dims: tuple
    type: str
    layout: str


@dataclass(frozen=True)
class STable:
    entries: int
    dims: tuple
    type: str
    layout: str


@dataclass(frozen=True)
class Ring:
    """Position p of slot s, head h at ((s * kv_heads + h) * length + p mod length) * head_dim (Graph.hs:137-143)."""

    slots: int
    kv_heads: int
    length: int
    head_dim: int


@dataclass(frozen=True)
class Paged:
    """Blocks from a pool listed per sequence in its block table (Graph.hs:144-152)."""

    blocks: int
    block_size: int
    kv_heads: int
    head_dim: int


CACHE_BF16 = "bf16"
CACHE_F16 = "f16"
CACHE_F32 = "f32"  # this target's addition: f32 caches for the f32 path


@dataclass(frozen=True)
class SCache:
    layout: object
    elem: str


@dataclass(frozen=True)
class Source:
    id: int
    name: str
    kind: object


def cache_kv_heads(layout) -> int:
    return layout.kv_heads


def cache_head_dim(layout) -> int:
    return layout.head_dim


# ---- operations ------------------------------------------------------------


@dataclass(frozen=True)
class RopeSpec:
    """Graph.hs:208-221: theta, the rotated pairs, the axes, the pairing (halves)."""

    theta: float
    rotated: int
    axes: int = 1
    pairs: str = "halves"


@dataclass(frozen=True)
class Reach:
    source: int
    ahead: int


@dataclass(frozen=True)
class AttnSpec:
    """Graph.hs:223-238."""

    heads: int
    kv_heads: int
    head_dim: int
    window: Optional[int]
    scale: float
    reach: Optional[Reach] = None


@dataclass(frozen=True)
class RouteSpec:
    k: int
    expert_scale: Optional[int]
    weights: str = "softmax_of_top_k"


@dataclass(frozen=True)
class StoreAt:
    cache: int
    positions: int
    sequences: int


@dataclass(frozen=True)
class AttendTo:
    keys: int
    values: int
    positions: int
    sequences: int


@dataclass(frozen=True)
class Op:
    """One operation (Graph.hs:299-360): `kind` names the constructor; the
    fields hold its arguments (value ids in `values`, source ids in `sources`)."""

    kind: str
    values: tuple = ()
    sources: tuple = ()
    args: tuple = ()


POINTWISE = {"Add", "GeluMul", "SiluMul", "ScaleBy", "Softcap", "KvStore"}


def op_values(op: Op) -> list:
    """The values an operation reads, in order (Graph.hs:362-381)."""
    return list(op.values)


def op_sources(op: Op) -> list:
    """The sources an operation reads or, for a cache, writes (Graph.hs:383-403)."""
    return list(op.sources)


@dataclass(frozen=True)
class Value:
    id: int
    name: str
    shape: Shape
    type: str


@dataclass(frozen=True)
class Node:
    id: int
    name: str
    op: Op
    outputs: tuple


@dataclass(frozen=True)
class Output:
    name: str
    value: int


@dataclass
class Program:
    name: str
    sources: list = field(default_factory=list)
    values: list = field(default_factory=list)
    nodes: list = field(default_factory=list)
    outputs: list = field(default_factory=list)

    def value(self, vid: int) -> Optional[Value]:
        return next((v for v in self.values if v.id == vid), None)

    def source(self, sid: int) -> Optional[Source]:
        return next((s for s in self.sources if s.id == sid), None)

    def node(self, nid: int) -> Optional[Node]:
        return next((n for n in self.nodes if n.id == nid), None)

    def producer_of(self, vid: int) -> Optional[Node]:
        return next((n for n in self.nodes if vid in n.outputs), None)


def _double(d: float) -> str:
    return "f64:0x" + format(struct.unpack("<Q", struct.pack("<d", d))[0], "x")


def render_program(p: Program) -> str:
    """A deterministic text form (Graph.hs:445-528)."""

    def shape(sh):
        return f"[{sh.width}/{sh.segment}]"

    def dims(ds):
        return "[" + ", ".join(str(d) for d in ds) + "]"

    def kind(k):
        if isinstance(k, SInput):
            return f"input {shape(k.shape)} {k.type}"
        if isinstance(k, SRowInts):
            return f"row_ints {k.count} below {k.bound}"
        if isinstance(k, SWeight):
            return f"weight {dims(k.dims)} {k.type} {k.layout}"
        if isinstance(k, STable):
            return f"table {k.entries} x {dims(k.dims)} {k.type} {k.layout}"
        if isinstance(k, SCache):
            lay = k.layout
            if isinstance(lay, Ring):
                t = f"ring slots {lay.slots} heads {lay.kv_heads} length {lay.length} dim {lay.head_dim}"
            else:
                t = f"paged blocks {lay.blocks} size {lay.block_size} heads {lay.kv_heads} dim {lay.head_dim}"
            return f"cache {t} {k.elem}"
        raise ValueError(k)

    def val(v):
        x = p.value(v)
        return x.name if x else f"%{v}"

    def src(s):
        x = p.source(s)
        return x.name if x else "?"

    def op(o: Op):
        k = o.kind
        if k == "Input":
            return f"input({src(o.sources[0])})"
        if k == "Linear":
            return f"linear({src(o.sources[0])}, {val(o.values[0])}) segment {o.args[0]}"
        if k == "LinearRouted":
            return f"linear_routed({src(o.sources[0])}, {val(o.values[0])}, {val(o.values[1])})"
        if k == "RmsNorm":
            eps, factor, gamma = o.args
            g = f", gamma {src(o.sources[0])}" if gamma else ""
            return f"rmsnorm({val(o.values[0])}, eps {_double(eps)}{g}, factor {_double(factor)})"
        if k in ("Add", "Concat"):
            return f"{k.lower()}({val(o.values[0])}, {val(o.values[1])})"
        if k == "ScaleBy":
            return f"scale_by({src(o.sources[0])}, {val(o.values[0])})"
        if k == "GatedGelu":
            return f"gated_gelu({val(o.values[0])})"
        if k == "GeluMul":
            return f"gelu_mul({val(o.values[0])}, {val(o.values[1])})"
        if k == "SiluMul":
            return f"silu_mul({val(o.values[0])}, {val(o.values[1])})"
        if k == "Rope":
            r = o.args[0]
            axes = "" if r.axes == 1 else f", axes {r.axes}"
            return f"rope({val(o.values[0])}, {src(o.sources[0])}, theta {_double(r.theta)}, rotated {r.rotated}{axes})"
        if k == "Softcap":
            return f"softcap({val(o.values[0])}, {_double(o.args[0])})"
        if k == "Route":
            r = o.args[0]
            sc = f", scale {src(r.expert_scale)}" if r.expert_scale is not None else ""
            return f"route({val(o.values[0])}, k {r.k}{sc})"
        if k == "CombineRanks":
            return f"combine_ranks({val(o.values[0])}, {val(o.values[1])})"
        if k == "KvStore":
            c, pos, slot = o.sources
            return f"kv_store({src(c)}, {src(pos)}, {src(slot)}, {val(o.values[0])})"
        if k == "Attend":
            a = o.args[0]
            kk, vv, pos, slot = o.sources[:4]
            w = f", window {a.window}" if a.window is not None else ""
            reach = f", reach {src(a.reach.source)} ahead {a.reach.ahead}" if a.reach else ""
            return (f"attend({', '.join([val(o.values[0]), src(kk), src(vv), src(pos), src(slot)])}, heads "
                    f"{a.heads}/{a.kv_heads}, dim {a.head_dim}{w}, scale {_double(a.scale)}{reach})")
        if k == "Gather":
            return f"gather({src(o.sources[0])}, {src(o.sources[1])}, factor {_double(o.args[0])})"
        if k == "Standardize":
            return f"standardize({val(o.values[0])}, {src(o.sources[0])}, {src(o.sources[1])}, factor {_double(o.args[0])})"
        if k == "ArgMax":
            return f"argmax({val(o.values[0])})"
        raise ValueError(k)

    lines = [f"program {p.name}"]
    lines += [f"  source {s.name} : {kind(s.kind)}" for s in p.sources]
    for n in p.nodes:
        outs = ", ".join(f"{val(v)} : {shape(p.value(v).shape)} {p.value(v).type}" for v in n.outputs)
        lines.append(f"  {outs}{' = ' if n.outputs else ''}{n.name} {op(n.op)}")
    lines += [f"  output {o.name} = {val(o.value)}" for o in p.outputs]
    return "".join(line + "\n" for line in lines)
