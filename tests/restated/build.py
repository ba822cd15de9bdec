"""Writing programs (src/FuryKernel/Program/Build.hs): a builder that
records sources, nodes and values in program order and hands back the
values to compute with. Sources keep their names; values and nodes take a
suffix where a name is taken (Build.hs:109-115)."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

from .graph import (
    CACHE_BF16,
    AttendTo,
    AttnSpec,
    Node,
    Op,
    Output,
    Program,
    RopeSpec,
    RouteSpec,
    SCache,
    SInput,
    Source,
    SRowInts,
    STable,
    StoreAt,
    SWeight,
    Shape,
    Value,
    whole_row,
)


@dataclass(frozen=True)
class Val:
    id: int
    shape: Shape


@dataclass(frozen=True)
class Src:
    id: int
    kind: object


class P:
    """A program being written: `program(name)` opens one, `done()` closes it."""

    def __init__(self, name: str):
        self.name = name
        self.names: set = set()
        self.sources: list = []
        self.values: list = []
        self.nodes: list = []
        self.outputs: list = []

    def done(self) -> Program:
        return Program(self.name, list(self.sources), list(self.values), list(self.nodes), list(self.outputs))

    # -- naming
    def _fresh(self, base: str) -> str:
        n, i = base, 1
        while n in self.names:
            n = f"{base}_{i}"
            i += 1
        self.names.add(n)
        return n

    def _source(self, name: str, kind) -> Src:
        s = Source(len(self.sources), name, kind)
        self.names.add(name)
        self.sources.append(s)
        return Src(s.id, kind)

    def _node(self, name: str, op: Op, outs: list) -> list:
        vals = []
        for vname, sh, t in outs:
            vn = self._fresh(vname)
            v = Value(len(self.values), vn, sh, t)
            self.values.append(v)
            vals.append((Val(v.id, sh), vn))
        nname = vals[0][1] if vals else self._fresh(name)
        self.nodes.append(Node(len(self.nodes), nname, op, tuple(v.id for v, _ in vals)))
        return [v for v, _ in vals]

    def _one(self, name: str, op: Op, sh: Shape, t: str = "f32") -> Val:
        return self._node(name, op, [(name, sh, t)])[0]

    # -- sources (Build.hs:153-199)
    def input(self, name: str, sh: Shape, t: str = "f32") -> Val:
        s = self._source(name, SInput(sh, t))
        v = Value(len(self.values), name, sh, t)
        self.values.append(v)
        self.nodes.append(Node(len(self.nodes), name, Op("Input", (), (s.id,)), (v.id,)))
        return Val(v.id, sh)

    def row_ints(self, name: str, n: int, bound: int) -> Src:
        return self._source(name, SRowInts(n, bound))

    def weight(self, name: str, dims: list, t: str = "bf16") -> Src:
        """A weight: the reference's `weight` is bf16 (Build.hs:175-176); this
        target's f32 path passes t = "f32", which the program gate takes
        (Program/Check.hs:105-119)."""
        dims = tuple(dims)
        return self._source(name, SWeight(dims, t, "out_in" if len(dims) == 2 else "row_major"))

    def rows_f32(self, name: str, dims: list) -> Src:
        return self._source(name, SWeight(tuple(dims), "f32", "row_major"))

    def table(self, name: str, n: int, dims: list, t: str = "bf16") -> Src:
        return self._source(name, STable(n, tuple(dims), t, "out_in"))

    def cache(self, name: str, layout, elem: str = CACHE_BF16) -> Src:
        return self._source(name, SCache(layout, elem))

    # -- operations (Build.hs:201-283)
    @staticmethod
    def _rows(s: Src) -> int:
        k = s.kind
        if isinstance(k, SWeight) and k.dims:
            return k.dims[0]
        if isinstance(k, STable) and k.dims:
            return k.dims[0]
        return 0

    def linear(self, name: str, w: Src, seg: int, x: Val) -> Val:
        n = self._rows(w)
        seg = n if seg == 0 else seg
        return self._one(name, Op("Linear", (x.id,), (w.id,), (seg,)), Shape(n, seg))

    def linear_routed(self, name: str, t: Src, ids: Val, x: Val) -> Val:
        n = self._rows(t)
        ranks = ids.shape.width
        return self._one(name, Op("LinearRouted", (ids.id, x.id), (t.id,)), Shape(ranks * n, n))

    def rmsnorm(self, name: str, eps: float, gamma: Optional[Src], factor: float, x: Val) -> Val:
        srcs = (gamma.id,) if gamma is not None else ()
        return self._one(name, Op("RmsNorm", (x.id,), srcs, (eps, factor, gamma is not None)), x.shape)

    def add(self, name: str, a: Val, b: Val) -> Val:
        return self._one(name, Op("Add", (a.id, b.id)), a.shape)

    def concatenate(self, name: str, a: Val, b: Val) -> Val:
        return self._one(name, Op("Concat", (a.id, b.id)), Shape(a.shape.width + b.shape.width, a.shape.segment))

    def scale_by(self, name: str, w: Src, x: Val) -> Val:
        return self._one(name, Op("ScaleBy", (x.id,), (w.id,)), x.shape)

    def gated_gelu(self, name: str, x: Val) -> Val:
        return self._one(name, Op("GatedGelu", (x.id,)), Shape(x.shape.width // 2, x.shape.segment // 2))

    def gelu_mul(self, name: str, a: Val, b: Val) -> Val:
        return self._one(name, Op("GeluMul", (a.id, b.id)), a.shape)

    def silu_mul(self, name: str, a: Val, b: Val) -> Val:
        """silu(a) * b elementwise: this target's addition, the SiLU-gated
        FFN's activation (the reference has GELU-tanh only, Graph.hs:322-327)."""
        return self._one(name, Op("SiluMul", (a.id, b.id)), a.shape)

    def rope(self, name: str, r: RopeSpec, pos: Src, x: Val) -> Val:
        return self._one(name, Op("Rope", (x.id,), (pos.id,), (r,)), x.shape)

    def softcap(self, name: str, c: float, x: Val) -> Val:
        return self._one(name, Op("Softcap", (x.id,), (), (c,)), x.shape)

    def route(self, name: str, k: int, scale: Optional[Src], x: Val):
        spec = RouteSpec(k, scale.id if scale is not None else None)
        srcs = (scale.id,) if scale is not None else ()
        ids, ws = self._node(name, Op("Route", (x.id,), srcs, (spec,)),
                             [(name + "_ids", whole_row(k), "u32"), (name + "_weights", whole_row(k), "f32")])
        return ids, ws

    def combine_ranks(self, name: str, w: Val, x: Val) -> Val:
        return self._one(name, Op("CombineRanks", (w.id, x.id)), whole_row(x.shape.segment))

    def kv_store(self, name: str, at: StoreAt, x: Val) -> None:
        self._node(name, Op("KvStore", (x.id,), (at.cache, at.positions, at.sequences)), [])

    def attend(self, name: str, spec: AttnSpec, q: Val, to: AttendTo) -> Val:
        srcs = (to.keys, to.values, to.positions, to.sequences) + ((spec.reach.source,) if spec.reach else ())
        return self._one(name, Op("Attend", (q.id,), srcs, (spec,)), q.shape)

    def gather(self, name: str, t: Src, tok: Src, factor: float) -> Val:
        width = t.kind.dims[1] if isinstance(t.kind, SWeight) and len(t.kind.dims) == 2 else 0
        return self._one(name, Op("Gather", (), (t.id, tok.id), (factor,)), whole_row(width))

    def standardize(self, name: str, b: Src, s: Src, factor: float, x: Val) -> Val:
        return self._one(name, Op("Standardize", (x.id,), (b.id, s.id), (factor,)), x.shape)

    def argmax(self, name: str, x: Val) -> Val:
        return self._one(name, Op("ArgMax", (x.id,)), whole_row(1), "u32")

    def output(self, name: str, v: Val) -> None:
        self.outputs.append(Output(name, v.id))


def program(name: str) -> P:
    return P(name)
