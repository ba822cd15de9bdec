"""The planner (src/FuryKernel/Program/Plan.hs): a program as steps, each one
kernel launch, and the cut points where steps meet.

No threadgroup waits for another inside a kernel: a value is stored once
the step that writes it has finished. Anchors (linear layers, attention)
set a step's grid; cheap operations are recomputed before them from stored
values or run as epilogues on a linear layer's tile; light steps hold cache
stores, attention's combine and outputs no anchor makes. The CUDA target
runs each step as one launch of a kernel from its table.

This restates the reference's rules, state machine and names, so that the
launch lists the target runs are the reference's plans (the golden plans of
test/Test/FuryKernel/ProgramTest.hs:559-640 hold here too:
tests/test_program.py).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

from .graph import POINTWISE, Program, Ring, SCache, SRowInts

# Costs (Plan.hs:196-206), ordered.
CHEAP, PASS, EXPENSIVE = 0, 1, 2


@dataclass(frozen=True)
class Work:
    """A node's part in a step (Plan.hs:124-139)."""

    kind: str  # Anchor, Recompute, Epilogue, Combine, Effect, Stage, Land
    node: int


@dataclass(frozen=True)
class Stored:
    """A value in memory between steps (Plan.hs:166-181): its elements of a
    type, attention's partials, or a staged store's values for a cache."""

    value: int
    form: tuple  # ("elements", type) | ("partials",) | ("staged", cache)


@dataclass
class Step:
    index: int
    name: str
    work: list
    stores: list
    reads: list
    caches: list

    def anchors(self) -> list:
        return [w.node for w in self.work if w.kind == "Anchor"]

    def is_light(self) -> bool:
        return not self.anchors()


@dataclass
class Plan:
    program: Program
    steps: list


@dataclass(frozen=True)
class PlanOptions:
    """Plan.hs:224-262."""

    horizontal: bool = True
    gated: bool = False
    store_gelus: bool = False
    sequence_rows: int = 1


DEFAULT = PlanOptions()


def anchor_family(op) -> Optional[str]:
    if op.kind in ("Linear", "LinearRouted"):
        return "Gemv"
    if op.kind == "Attend":
        return "Attention"
    return None


def node_cost(p: Program, op) -> int:
    """Plan.hs:214-223."""
    if op.kind in ("RmsNorm", "Route", "ArgMax"):
        return PASS
    if op.kind == "Gather":
        s = p.source(op.sources[1])
        if s is not None and isinstance(s.kind, SRowInts) and s.kind.count > 1:
            return EXPENSIVE
    return CHEAP


def ring_room(length: int, window: Optional[int], bound: int) -> int:
    """Plan.hs:270-281."""
    seen = window if window is not None else bound
    return 0 if seen > length else length - seen + 1


@dataclass
class _StepB:
    index: int
    work: list = field(default_factory=list)
    stores: list = field(default_factory=list)
    family: Optional[str] = None
    writes: set = field(default_factory=set)


class _Planner:
    def __init__(self, opts: PlanOptions, p: Program):
        self.o, self.p = opts, p
        self.avail: dict = {}
        self.closed: list = []
        self.open: Optional[_StepB] = None
        self.next = 0
        self.landing: list = []
        self.nodes = {n.id: n for n in p.nodes}
        self.producer = {v: n for n in p.nodes for v in n.outputs}
        self.consumers: dict = {}
        for n in p.nodes:
            for v in n.op.values:
                self.consumers.setdefault(v, []).append(n.id)
        self.output_values = {o.value for o in p.outputs}
        self.staged = self._staged()

    # -- the program's facts
    def op_of(self, n):
        return self.nodes[n].op

    def type_of(self, v):
        val = self.p.value(v)
        return val.type if val else "f32"

    def outs_of(self, n):
        return list(self.nodes[n].outputs) if n in self.nodes else []

    def _position_bound(self, s):
        src = self.p.source(s)
        return src.kind.bound if src is not None and isinstance(src.kind, SRowInts) else 0

    def _staged(self) -> set:
        out = set()
        nodes = self.p.nodes
        for i, n in enumerate(nodes):
            if n.op.kind != "KvStore":
                continue
            c = n.op.sources[0]
            src = self.p.source(c)
            if src is None or not isinstance(src.kind, SCache) or not isinstance(src.kind.layout, Ring):
                continue
            length = src.kind.layout.length
            for r in nodes[i + 1:]:
                if r.op.kind == "Attend" and c in r.op.sources[:2]:
                    a = r.op.args[0]
                    if self.o.sequence_rows > ring_room(length, a.window, self._position_bound(r.op.sources[2])):
                        out.add(n.id)
                        break
        return out

    def staged_into(self, c):
        for n in self.p.nodes:
            if n.op.kind == "KvStore" and n.op.sources[0] == c and n.id in self.staged:
                return n.id
        return None

    def last_reader(self, c):
        readers = [n.id for n in self.p.nodes if n.op.kind == "Attend" and c in n.op.sources[:2]]
        return readers[-1] if readers else None

    # -- availability
    def avail_of(self, v):
        return self.avail.get(v, ("stored", -1))

    def open_index(self):
        return self.open.index if self.open is not None else None

    # -- steps
    def close_open(self):
        if self.open is None:
            return
        self.outputs_here()
        self.store_shared()
        sb = self.open
        in_step = {w.node for w in sb.work}
        tiled = [v for w in sb.work if w.kind in ("Anchor", "Epilogue") for v in self.outs_of(w.node)]
        stores = []
        for v in tiled:
            stores += self.store_tile(sb, in_step, v)
        sb.stores = sb.stores + stores
        self.closed.append(sb)
        self.open = None

    def store_tile(self, sb, in_step, v):
        outside = any(c not in in_step for c in self.consumers.get(v, []))
        if not (outside or v in self.output_values):
            return []
        n = self.producer.get(v)
        if n is not None and n.op.kind == "Attend":
            self.avail[v] = ("partials", sb.index)
            return [Stored(v, ("partials",))]
        self.avail[v] = ("stored", sb.index)
        return [Stored(v, ("elements", self.type_of(v)))]

    def new_step(self, fam):
        self.close_open()
        sb = _StepB(self.next, family=fam)
        self.open = sb
        self.next += 1
        return sb

    def light_step(self):
        sb = self.open
        if not (sb is not None and sb.family is None and not any(w.kind == "Anchor" for w in sb.work)):
            self.new_step(None)
        i = self.open_index()
        due = [l for l in self.landing if i is not None and i > l[0]]
        for _, n, c in due:
            self.add_work(Work("Land", n))
            if self.open is not None:
                self.open.writes.add(c)
        self.landing = [l for l in self.landing if l not in due]

    def land_rest(self):
        if self.landing:
            self.light_step()

    def add_work(self, w: Work):
        if self.open is not None and w.node not in [x.node for x in self.open.work]:
            self.open.work.append(w)

    def add_store(self, st: Stored):
        if self.open is not None and st not in self.open.stores:
            self.open.stores.append(st)

    # -- chains
    def chain(self, v):
        a = self.avail_of(v)
        i = self.open_index()
        n = self.producer.get(v)
        if a[0] == "stored" and a[1] != i:
            return
        if a[0] == "partials" and n is not None and a[1] != i:
            self.add_work(Work("Combine", n.id))
            return
        if n is not None:
            planned = self.open is not None and n.id in [w.node for w in self.open.work]
            if not planned:
                for u in n.op.values:
                    self.chain(u)
                self.add_work(Work("Recompute", n.id))

    def outputs_here(self):
        st = self.open
        if st is None:
            return
        combined = {w.node for w in st.work if w.kind == "Combine"}

        def has(v):
            a = self.avail_of(v)
            if a[0] == "stored":
                return True
            if a[0] == "partials":
                n = self.producer.get(v)
                return n is not None and n.id in combined
            if a[0] == "virtual":
                n = self.producer.get(v)
                if n is not None:
                    return all(has(u) for u in n.op.values)
            return False

        if st.family is None and combined:
            for o in self.p.outputs:
                if self.avail_of(o.value)[0] == "virtual" and has(o.value):
                    self.materialize(o.value)

    def store_shared(self):
        st = self.open
        if st is None:
            return
        in_step = {w.node for w in st.work}

        def needed(v):
            return any(c not in in_step for c in self.consumers.get(v, [])) or v in self.output_values

        def store(v):
            self.add_store(Stored(v, ("elements", self.type_of(v))))
            self.avail[v] = ("stored", st.index)

        for n in [w.node for w in st.work if w.kind == "Recompute"]:
            for v in self.outs_of(n):
                a = self.avail_of(v)
                if a[0] == "virtual" and a[1] >= PASS and needed(v):
                    store(v)
        for n in [w.node for w in st.work if w.kind == "Combine"]:
            for v in self.outs_of(n):
                if self.avail_of(v)[0] == "partials" and needed(v):
                    store(v)

    def materialize(self, v):
        self.light_step()
        self.chain(v)
        i = self.open_index()
        if i is not None:
            self.add_store(Stored(v, ("elements", self.type_of(v))))
            self.avail[v] = ("stored", i)

    # -- nodes
    def node(self, n):
        op = n.op
        if op.kind == "Input":
            for v in n.outputs:
                self.avail[v] = ("stored", -1)
        elif anchor_family(op) is not None:
            self.anchor(n, anchor_family(op))
        elif op.kind == "KvStore":
            self.effect(n)
        else:
            self.light(n)

    def anchor(self, n, fam):
        op = n.op
        ins = list(op.values)
        if any(self.touches_open(v) for v in ins):
            self.close_open()
        for v in ins:
            if self.expensive(v) or self.stored_gelu(v):
                self.materialize(v)
        if op.kind == "LinearRouted" and self.o.gated:
            if self.avail_of(op.values[0])[0] != "stored":
                self.materialize(op.values[0])
        sb = self.open
        reads_caches = [c for c in op.sources if sb is not None and c in sb.writes]
        gated_here = op.kind == "LinearRouted" and self.o.gated
        joins = (sb is not None and self.o.horizontal and sb.family == fam and not reads_caches and not gated_here)
        if not joins:
            self.new_step(fam)
        for v in ins:
            self.chain(v)
        self.add_work(Work("Anchor", n.id))
        s = self.open_index()
        if s is not None:
            for v in n.outputs:
                self.avail[v] = ("partials", s) if op.kind == "Attend" else ("tile", s, n.id)
            if op.kind == "Attend":
                k, vv = op.sources[0], op.sources[1]
                for c in dict.fromkeys([k, vv]):
                    store = self.staged_into(c)
                    if self.last_reader(c) == n.id and store is not None:
                        self.landing.append((s, store, c))

    def touches_open(self, v0) -> bool:
        i = self.open_index()
        seen = set()
        todo = [v0]
        while todo:
            v = todo.pop(0)
            if v in seen:
                continue
            seen.add(v)
            a = self.avail_of(v)
            if a[0] in ("tile", "partials") and a[1] == i:
                return True
            if a[0] == "virtual":
                n = self.producer.get(v)
                if n is not None:
                    todo = list(n.op.values) + todo
        return False

    def stored_gelu(self, v) -> bool:
        if not self.o.store_gelus:
            return False
        n = self.producer.get(v)
        return n is not None and n.op.kind in ("GeluMul", "GatedGelu") and self.avail_of(v)[0] == "virtual"

    def expensive(self, v) -> bool:
        a = self.avail_of(v)
        return a[0] == "partials" or (a[0] == "virtual" and a[1] >= EXPENSIVE)

    def input_cost(self, v) -> int:
        a = self.avail_of(v)
        if a[0] == "virtual":
            return a[1]
        if a[0] == "partials":
            return EXPENSIVE
        return CHEAP

    def light(self, n):
        op = n.op
        ins = list(op.values)
        avails = [self.avail_of(v) for v in ins]
        i = self.open_index()
        on_tile = [(v, a[2]) for v, a in zip(ins, avails) if a[0] == "tile" and a[1] == i]
        anchors = list(dict.fromkeys(a for _, a in on_tile))
        tiled_vals = [v for v, _ in on_tile]

        def other(v, a):
            if a[0] == "stored":
                return True
            if a[0] == "virtual" and a[1] == CHEAP:
                return not self.touches_open(v)
            return False

        others_ok = all(other(v, a) for v, a in zip(ins, avails) if v not in tiled_vals)
        if len(anchors) == 1 and op.kind in POINTWISE and others_ok:
            for v, a in zip(ins, avails):
                if a[0] == "virtual":
                    self.chain(v)
            self.add_work(Work("Epilogue", n.id))
            if i is not None:
                for v in n.outputs:
                    self.avail[v] = ("tile", i, anchors[0])
        else:
            c = max([node_cost(self.p, op)] + [self.input_cost(v) for v in ins])
            for v in n.outputs:
                self.avail[v] = ("virtual", c)
            if self.o.gated and (self._feeds_routed(n) or self._routes_output(n)):
                if any(self.touches_open(v) for v in ins):
                    self.close_open()
                for v in n.outputs[:1]:
                    self.materialize(v)

    def _feeds_routed(self, r) -> bool:
        if r.op.kind != "Route":
            return False
        for v in r.outputs[:1]:
            for c in self.consumers.get(v, []):
                op = self.op_of(c)
                if op.kind == "LinearRouted" and op.values[0] == v:
                    return True
        return False

    def _routes_output(self, r) -> bool:
        return r.op.kind == "Route" and any(v in self.output_values for v in r.outputs[:1])

    def effect(self, n):
        op = n.op
        ins = list(op.values)
        if n.id in self.staged:
            self.light_step()
            for v in ins:
                self.chain(v)
            self.add_work(Work("Stage", n.id))
            self.add_store(Stored(op.values[0], ("staged", op.sources[0])))
            return
        avails = [self.avail_of(v) for v in ins]
        i = self.open_index()
        on_tile = [v for v, a in zip(ins, avails) if a[0] == "tile" and a[1] == i]
        if on_tile and op.kind in POINTWISE and len(on_tile) == len(ins):
            self.add_work(Work("Epilogue", n.id))
        else:
            self.light_step()
            for v in ins:
                self.chain(v)
            self.add_work(Work("Effect", n.id))
        if self.open is not None:
            self.open.writes.add(op.sources[0])

    def outputs(self):
        for o in self.p.outputs:
            if self.avail_of(o.value)[0] in ("virtual", "partials"):
                self.materialize(o.value)

    # -- the steps as the plan gives them
    def finish(self, sb) -> Step:
        return Step(sb.index, self.name(sb), sorted(sb.work, key=lambda w: w.node),
                    sorted(sb.stores, key=lambda s: s.value), sorted(self.reads_of(sb), key=lambda s: s.value),
                    list(dict.fromkeys(c for w in sb.work for c in self.caches(w))))

    def caches(self, w):
        if w.kind in ("Stage", "Combine"):
            return []
        op = self.op_of(w.node)
        if op.kind == "KvStore":
            return [op.sources[0]]
        if op.kind == "Attend":
            return [op.sources[0], op.sources[1]]
        return []

    def reads_of(self, sb):
        making = {"Combine", "Anchor", "Recompute", "Epilogue"}
        in_step = {v for w in sb.work if w.kind in making for v in self.outs_of(w.node)}

        def wanted(w, form):
            if w.kind == "Combine":
                return form[0] == "partials"
            return form[0] == "elements"

        def stages_read(w):
            op = self.op_of(w.node)
            if w.kind == "Anchor" and op.kind == "Attend":
                return list(dict.fromkeys([op.sources[0], op.sources[1]]))
            if w.kind == "Land" and op.kind == "KvStore":
                return [op.sources[0]]
            return []

        def reads_of_work(w):
            if w.kind == "Combine":
                return self.outs_of(w.node)
            if w.kind == "Land":
                return []
            return [v for v in self.op_of(w.node).values if v not in in_step]

        out = []
        for w in sb.work:
            for v in reads_of_work(w):
                for st in self.stored_before(sb.index, v):
                    if wanted(w, st.form) and st not in out:
                        out.append(st)
        for w in sb.work:
            for c in stages_read(w):
                for st in self.staged_before(sb.index, c):
                    if st not in out:
                        out.append(st)
        return out

    def stored_before(self, s, v):
        out = [st for sb in self.closed if sb.index < s for st in sb.stores if st.value == v]
        n = self.producer.get(v)
        if n is not None and n.op.kind == "Input":
            out.append(Stored(v, ("elements", self.type_of(v))))
        return out

    def staged_before(self, s, c):
        return [st for sb in self.closed if sb.index < s for st in sb.stores if st.form == ("staged", c)]

    def name(self, sb) -> str:
        anchors = [self.op_of(w.node) for w in sb.work if w.kind == "Anchor"]
        if anchors:
            words = list(dict.fromkeys("attend" if op.kind == "Attend" else "gemv" for op in anchors))
            return f"s{sb.index}_" + "_".join(words)
        for w in sb.work:
            if w.kind in ("Effect", "Stage"):
                return f"s{sb.index}_store"
            if w.kind == "Combine":
                return f"s{sb.index}_combine"
            if w.kind == "Recompute":
                els = [st for st in sb.stores if st.form[0] == "elements"]
                if els:
                    return f"s{sb.index}_" + self.p.value(els[0].value).name
        if any(w.kind == "Land" for w in sb.work):
            return f"s{sb.index}_land"
        return f"s{sb.index}_light"

    def run(self) -> Plan:
        for n in self.p.nodes:
            self.node(n)
        self.outputs()
        self.land_rest()
        self.close_open()
        return Plan(self.p, [self.finish(sb) for sb in self.closed])


def plan(opts: PlanOptions, p: Program) -> Plan:
    """plan :: PlanOptions -> CheckedProgram -> Plan (Plan.hs:314-318)."""
    return _Planner(opts, p).run()


def render_plan(pl: Plan) -> str:
    """A deterministic text form (Plan.hs:815-843)."""
    p = pl.program

    def stored(st):
        name = p.value(st.value).name
        if st.form[0] == "elements":
            return f"{name} {st.form[1]}"
        if st.form[0] == "partials":
            return f"{name} partials"
        return f"{name} staged for {p.source(st.form[1]).name}"

    lines = [f"plan {p.name}"]
    for s in pl.steps:
        lines.append(f"  step {s.name}")
        for w in s.work:
            lines.append(f"    {w.kind.lower()} {p.node(w.node).name}")
        lines += [f"    reads {stored(st)}" for st in s.reads]
        lines += [f"    stores {stored(st)}" for st in s.stores]
    return "".join(line + "\n" for line in lines)


def is_step_name(t: str) -> bool:
    """src/FuryKernel/Program/Plan.hs:162-165."""
    if not t.startswith("s"):
        return False
    rest = t[1:]
    digits = 0
    while digits < len(rest) and rest[digits].isdigit():
        digits += 1
    return digits > 0 and rest[digits:].startswith("_") and len(rest[digits:]) > 1
