"""The launch sequence of planned programs on the device.

A plan's steps (src/FuryKernel/Program/Plan.hs:109-121) become one launch
each of a kernel in the target's table: the step's anchors set the kernel,
its recomputed operations become the kernel's prologue and its epilogues
the kernel's epilogue. The step shapes of the Llama-shaped programs
(furykernel_b200.program.llama) are the ones lowered; any other step shape
is refused with the step's text.

Memory: a stored value lives in a device buffer of its rows; the anchors of
one step (horizontal q/k/v, gate/up) write adjacent columns of one buffer,
and their weights lie adjacent in the weight arena, so the step is one GEMV
over the concatenated rows. KV caches are Ring arenas per layer.

`Llama` builds a whole decode step -- the embedding gather, every layer's
plan, the head's plan -- captures it as one CUDA graph, and replays it per
step: host token ids in, greedy ids out. Its launch list comes from the C++
host library (libfurykernel_host.so: the same programs, planner and
lowering); `lower_step` and `Llama._launches_restated` state the same
algorithm in Python, and the tests hold the library to them launch for
launch.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

from . import _native as N
from .program import plan as PL
from .program.graph import Paged, SCache, SRowInts, SWeight
from .program.llama import LlamaShape, embed_program, head_program, layer_program
from .target import CACHE_SUFFIX, WEIGHT_SUFFIX


class Unlowerable(N.Refused):
    """A step whose shape no kernel of the target runs."""


@dataclass
class View:
    """A stored value: its buffer, its first column and the buffer's row stride."""

    buf: object  # DeviceBuffer or int address
    col: int
    ld: int
    width: int

    @property
    def base(self) -> int:
        return self.buf.ptr if isinstance(self.buf, N.DeviceBuffer) else int(self.buf)

    @property
    def ptr(self) -> int:
        return self.base + 4 * self.col


@dataclass
class Launch:
    kernel: str
    params: dict
    bufs: list

    def run(self, ctx: N.Context) -> None:
        ctx.launch(self.kernel, self.params, self.bufs)


@dataclass
class Binding:
    """What a program's sources and stored values are on the device."""

    weights: dict = field(default_factory=dict)  # source name -> address
    ints: dict = field(default_factory=dict)  # source name -> address of [m] u32
    caches: dict = field(default_factory=dict)  # source name -> address of the layer's Ring
    values: dict = field(default_factory=dict)  # value name -> View
    m: int = 1


def _work_text(p, step) -> str:
    return "; ".join(f"{w.kind.lower()} {p.node(w.node).name}" for w in step.work)


# A kernel's element-type form: the f32 entry's name, or with the suffix of
# its 16-bit weights or its 16-bit KV caches (target.WEIGHT_SUFFIX,
# target.CACHE_SUFFIX).
def kernel_form(kernel: str) -> tuple:
    """(the f32 entry's name, the suffix of the form)."""
    for suffix in ("_wbf16", "_wf16", "_kvbf16", "_kvf16"):
        if kernel.endswith(suffix):
            return kernel[:-len(suffix)], suffix
    return kernel, ""


def _weight_suffix(step, t: str) -> str:
    if t in WEIGHT_SUFFIX:
        return WEIGHT_SUFFIX[t]
    raise Unlowerable(N.FKC_ERR_ARGUMENT, f"{step.name}: no kernel reads {t} weights.")


def _cache_suffix(step, elem: str) -> str:
    if elem in CACHE_SUFFIX:
        return CACHE_SUFFIX[elem]
    raise Unlowerable(N.FKC_ERR_ARGUMENT, f"{step.name}: no kernel reads {elem} caches.")


def lower_step(p, step, b: Binding, tables: dict, attn: dict) -> Launch:
    """One step of a plan as one launch (the step shapes of the Llama plans)."""
    work = [(w.kind, p.node(w.node)) for w in step.work]
    anchors = [n for k, n in work if k == "Anchor"]
    recomputed = {n.outputs[0]: n for k, n in work if k == "Recompute"}
    epilogues = [n for k, n in work if k == "Epilogue"]
    vname = lambda v: p.value(v).name  # noqa: E731

    def stored(v) -> View:
        view = b.values.get(vname(v))
        if view is None:
            raise Unlowerable(N.FKC_ERR_ARGUMENT, f"{step.name}: {vname(v)} is not stored where the step reads it.")
        return view

    if anchors and all(n.op.kind == "Linear" for n in anchors):
        x_id = anchors[0].op.values[0]
        if any(n.op.values[0] != x_id for n in anchors):
            raise Unlowerable(N.FKC_ERR_ARGUMENT, f"{step.name}: anchors of different inputs: {_work_text(p, step)}")
        ws = [p.source(n.op.sources[0]) for n in anchors]
        if any(w.kind.type != ws[0].kind.type for w in ws):
            raise Unlowerable(N.FKC_ERR_ARGUMENT, f"{step.name}: its anchors' weights differ in type.")
        wt = _weight_suffix(step, ws[0].kind.type)
        esz = 2 if wt else 4
        w0 = b.weights[ws[0].name]
        n_total = sum(w.kind.dims[0] for w in ws)
        k = ws[0].kind.dims[1]
        addr = w0
        for w in ws:  # the anchors' weights must lie adjacent
            if b.weights[w.name] != addr:
                raise Unlowerable(N.FKC_ERR_ARGUMENT, f"{step.name}: the weights of its anchors are not adjacent.")
            addr += esz * w.kind.dims[0] * k
        if epilogues:
            (ep,) = epilogues
            if ep.op.kind != "Add" or len(anchors) != 1:
                raise Unlowerable(N.FKC_ERR_ARGUMENT, f"{step.name}: epilogue {ep.name} is not one residual add.")
            tile = anchors[0].outputs[0]
            r_id = ep.op.values[0] if ep.op.values[1] == tile else ep.op.values[1]
            y = stored(ep.outputs[0])
        else:
            y = b.values[vname(anchors[0].outputs[0])]
            for n in anchors[1:]:  # adjacent columns
                nxt = b.values[vname(n.outputs[0])]
                if nxt.buf is not y.buf:
                    raise Unlowerable(N.FKC_ERR_ARGUMENT, f"{step.name}: its anchors' outputs are not adjacent.")
        split = attn.get("split", 1)
        base = {"n": n_total, "k": k, "m": b.m, "split": split, "ldy": y.ld}
        xn = recomputed.get(x_id)
        if xn is None:
            x = stored(x_id)
            base["ldx"] = x.ld
            if epilogues:
                r = stored(r_id)
                return Launch("gemv_add" + wt, dict(base, ldr=r.ld), [w0, x.ptr, r.ptr, y.ptr])
            return Launch("gemv" + wt, base, [w0, x.ptr, y.ptr])
        if xn.op.kind == "RmsNorm" and not epilogues:
            eps, factor, has_gamma = xn.op.args
            x = stored(xn.op.values[0])
            g = p.source(xn.op.sources[0])
            if g.kind.type != ws[0].kind.type:
                raise Unlowerable(N.FKC_ERR_ARGUMENT, f"{step.name}: the norm's gain and the weights differ in type.")
            gamma = b.weights[g.name]
            return Launch("gemv_rmsnorm" + wt, dict(base, ldx=x.ld, eps=eps, factor=factor),
                          [w0, x.ptr, gamma, y.ptr])
        if xn.op.kind == "SiluMul":
            g, u = (stored(v) for v in xn.op.values)
            if g.buf is not u.buf or g.ld != u.ld:
                raise Unlowerable(N.FKC_ERR_ARGUMENT, f"{step.name}: SiLU-gate's halves are not one row.")
            base = dict(base, ldx=g.ld, up_off=u.col - g.col)
            if epilogues:
                r = stored(r_id)
                return Launch("gemv_silu_add" + wt, dict(base, ldr=r.ld), [w0, g.ptr, r.ptr, y.ptr])
            return Launch("gemv_silu" + wt, base, [w0, g.ptr, y.ptr])
        raise Unlowerable(N.FKC_ERR_ARGUMENT, f"{step.name}: no kernel runs {_work_text(p, step)}")

    if len(anchors) == 1 and anchors[0].op.kind == "Attend":
        att = anchors[0]
        spec = att.op.args[0]
        qn = recomputed.get(att.op.values[0])
        if qn is None or qn.op.kind != "Rope":
            raise Unlowerable(N.FKC_ERR_ARGUMENT, f"{step.name}: attention without its query's rotation.")
        q = stored(qn.op.values[0])
        kc, vc, pos, slot = (p.source(s).name for s in att.op.sources[:4])
        layout = p.source(att.op.sources[0]).kind.layout
        ct = _cache_suffix(step, p.source(att.op.sources[0]).kind.elem)
        part = attn["partials"]
        if isinstance(layout, Paged):  # through the rows' block tables
            return Launch("attend_split_paged" + ct,
                          {"m": b.m, "heads": spec.heads, "kv_heads": spec.kv_heads, "d": spec.head_dim,
                           "block_size": layout.block_size, "table_len": p.source(att.op.sources[3]).kind.count,
                           "blocks": layout.blocks, "rotated": qn.op.args[0].rotated, "chunk": attn["chunk"],
                           "max_splits": attn["max_splits"], "ldq": q.ld, "q_off": q.col, "scale": spec.scale},
                          [q.base, tables["cos"], tables["sin"], b.ints[pos], b.ints[slot],
                           b.caches[kc], b.caches[vc], part[0], part[1], part[2]])
        return Launch("attend_split" + ct,
                      {"m": b.m, "heads": spec.heads, "kv_heads": spec.kv_heads, "d": spec.head_dim,
                       "length": layout.length, "rotated": qn.op.args[0].rotated, "chunk": attn["chunk"],
                       "max_splits": attn["max_splits"], "ldq": q.ld, "q_off": q.col, "scale": spec.scale},
                      [q.base, tables["cos"], tables["sin"], b.ints[pos], b.ints[slot],
                       b.caches[kc], b.caches[vc], part[0], part[1], part[2]])

    kinds = [k for k, _ in work]
    if kinds == ["Combine"]:
        att = work[0][1]
        spec = att.op.args[0]
        out = stored(att.outputs[0])
        pos = p.source(att.op.sources[2]).name
        part = attn["partials"]
        return Launch("attend_combine",
                      {"m": b.m, "heads": spec.heads, "d": spec.head_dim, "chunk": attn["chunk"],
                       "max_splits": attn["max_splits"], "ldo": out.ld},
                      [part[0], part[1], part[2], b.ints[pos], out.ptr])

    effects = [n for k, n in work if k == "Effect"]
    if effects and all(n.op.kind == "KvStore" for n in effects) and len(effects) == 2:
        sk, sv = effects
        kn = recomputed.get(sk.op.values[0])
        if kn is None or kn.op.kind != "Rope":
            raise Unlowerable(N.FKC_ERR_ARGUMENT, f"{step.name}: keys stored without their rotation.")
        kview, vview = stored(kn.op.values[0]), stored(sv.op.values[0])
        if kview.buf is not vview.buf:
            raise Unlowerable(N.FKC_ERR_ARGUMENT, f"{step.name}: keys and values are not one row.")
        layout = p.source(sk.op.sources[0]).kind.layout
        ct = _cache_suffix(step, p.source(sk.op.sources[0]).kind.elem)
        pos, slot = (p.source(s).name for s in sk.op.sources[1:3])
        if isinstance(layout, Paged):  # through the rows' block tables
            return Launch("kv_store_paged" + ct,
                          {"m": b.m, "kv_heads": layout.kv_heads, "d": layout.head_dim,
                           "block_size": layout.block_size, "table_len": p.source(sk.op.sources[2]).kind.count,
                           "blocks": layout.blocks, "rotated": kn.op.args[0].rotated, "ldq": kview.ld,
                           "k_off": kview.col, "v_off": vview.col},
                          [kview.base, tables["cos"], tables["sin"], b.ints[pos], b.ints[slot],
                           b.caches[p.source(sk.op.sources[0]).name], b.caches[p.source(sv.op.sources[0]).name]])
        return Launch("kv_store_ring" + ct,
                      {"m": b.m, "kv_heads": layout.kv_heads, "d": layout.head_dim, "length": layout.length,
                       "rotated": kn.op.args[0].rotated, "ldq": kview.ld, "k_off": kview.col, "v_off": vview.col},
                      [kview.base, tables["cos"], tables["sin"], b.ints[pos], b.ints[slot],
                       b.caches[p.source(sk.op.sources[0]).name], b.caches[p.source(sv.op.sources[0]).name]])

    if kinds == ["Recompute"] and work[0][1].op.kind == "Gather":
        g = work[0][1]
        table, tok = (p.source(s) for s in g.op.sources)
        y = stored(g.outputs[0])
        return Launch("gather" + _weight_suffix(step, table.kind.type),
                      {"width": table.kind.dims[1], "m": b.m, "factor": g.op.args[0]},
                      [b.weights[table.name], b.ints[tok.name], y.ptr])

    if kinds == ["Recompute"] and work[0][1].op.kind == "ArgMax":
        a = work[0][1]
        x = stored(a.op.values[0])
        y = stored(a.outputs[0])
        return Launch("argmax", {"m": b.m, "n": x.width, "ldx": x.ld}, [x.ptr, y.ptr])

    raise Unlowerable(N.FKC_ERR_ARGUMENT, f"{step.name}: no kernel runs {_work_text(p, step)}")


def lower_steps(p, step, b: Binding, tables: dict, attn: dict) -> list:
    """One step of a plan as its launches: the routed-experts steps as
    several (their parts run as separate kernels), any other as
    lower_step's one."""
    work = [(w.kind, p.node(w.node)) for w in step.work]
    kinds = sorted((k, n.op.kind) for k, n in work)
    vname = lambda v: p.value(v).name  # noqa: E731

    def stored(v) -> View:
        view = b.values.get(vname(v))
        if view is None:
            raise Unlowerable(N.FKC_ERR_ARGUMENT, f"{step.name}: {vname(v)} is not stored where the step reads it.")
        return view

    def node(kind):
        return next(n for _, n in work if n.op.kind == kind)

    stored_values = {st.value for st in step.stores}
    if kinds == [("Anchor", "Linear"), ("Recompute", "RmsNorm")] and node("RmsNorm").outputs[0] in stored_values:
        # The norm's row is stored for a later step: the rows, then the GEMV of them.
        nn, lin = node("RmsNorm"), node("Linear")
        eps, factor, _ = nn.op.args
        x, y, out = stored(nn.op.values[0]), stored(nn.outputs[0]), stored(lin.outputs[0])
        if x.ld != x.width or y.ld != y.width:
            raise Unlowerable(N.FKC_ERR_ARGUMENT, f"{step.name}: a stored norm of rows that are not whole.")
        w = p.source(lin.op.sources[0])
        wt = _weight_suffix(step, w.kind.type)
        n, k = w.kind.dims
        return [Launch("rmsnorm_rows" + wt, {"rows": b.m, "h": x.width, "eps": eps, "factor": factor},
                       [x.ptr, b.weights[p.source(nn.op.sources[0]).name], y.ptr]),
                Launch("gemv" + wt, {"n": n, "k": k, "m": b.m, "split": attn.get("split", 1), "ldx": y.ld,
                                     "ldy": out.ld}, [b.weights[w.name], y.ptr, out.ptr])]
    # Routed experts: the route, the GELU gate and the routed GEMV, each a
    # step of its own (the gated plan's, Plan.hs:246-251, with or without
    # stored gelus) or the route or the gate recomputed in the GEMV's step.
    routed_shapes = ([("Recompute", "Route")], [("Recompute", "GatedGelu")], [("Anchor", "LinearRouted")],
                     [("Anchor", "LinearRouted"), ("Recompute", "Route")],
                     [("Anchor", "LinearRouted"), ("Recompute", "GatedGelu")])
    if kinds in routed_shapes:
        ops = {op for _, op in kinds}
        out = []
        if "Route" in ops:
            r = node("Route")
            logits, ids, ws = stored(r.op.values[0]), stored(r.outputs[0]), stored(r.outputs[1])
            params = {"m": b.m, "n": logits.width, "k": ids.width, "ldx": logits.ld}
            if r.op.args[0].expert_scale is not None:  # each expert's weight times its scale
                sc = p.source(r.op.args[0].expert_scale)
                out.append(Launch("route_topk_scaled" + _weight_suffix(step, sc.kind.type), params,
                                  [logits.ptr, b.weights[sc.name], ids.ptr, ws.ptr]))
            else:
                out.append(Launch("route_topk", params, [logits.ptr, ids.ptr, ws.ptr]))
        if "GatedGelu" in ops:
            g = node("GatedGelu")
            gu, x = stored(g.op.values[0]), stored(g.outputs[0])
            f = p.value(g.outputs[0]).shape.segment
            if gu.ld != gu.width or x.ld != x.width:
                raise Unlowerable(N.FKC_ERR_ARGUMENT, f"{step.name}: a gate of rows that are not whole.")
            if f == 0 or x.width % f:
                raise Unlowerable(N.FKC_ERR_ARGUMENT, f"{step.name}: a gate whose rows are not whole segments.")
            out.append(Launch("gated_gelu", {"segments": b.m * (x.width // f), "f": f}, [gu.ptr, x.ptr]))
        if "LinearRouted" in ops:
            lr = node("LinearRouted")
            t = p.source(lr.op.sources[0])
            tsuf = _weight_suffix(step, t.kind.type)
            n, kk = t.kind.dims
            ids_v, x_id = lr.op.values
            ids, x, y = stored(ids_v), stored(x_id), stored(lr.outputs[0])
            out.append(Launch("gemv_routed" + tsuf, {"entries": t.kind.entries, "n": n, "kk": kk, "m": b.m,
                                                     "k": ids.width, "split": attn.get("split", 1), "ldx": x.ld,
                                                     "ldy": y.ld, "per_rank": int(x.width != kk)},
                              [b.weights[t.name], ids.ptr, x.ptr, y.ptr]))
        return out
    if kinds == [("Recompute", "Add"), ("Recompute", "CombineRanks")]:
        c, a = node("CombineRanks"), node("Add")
        ws, segs, y = stored(c.op.values[0]), stored(c.op.values[1]), stored(a.outputs[0])
        r_id = a.op.values[0] if a.op.values[1] == c.outputs[0] else a.op.values[1]
        r = stored(r_id)
        if any(v.ld != v.width for v in (ws, segs, y, r)):
            raise Unlowerable(N.FKC_ERR_ARGUMENT, f"{step.name}: a combine of rows that are not whole.")
        return [Launch("combine_ranks_add", {"m": b.m, "k": ws.width, "d": y.width}, [r.ptr, ws.ptr, segs.ptr, y.ptr])]
    return [lower_step(p, step, b, tables, attn)]


def split_for(n_rows: int, k: int, sms: int) -> int:
    """Split-K for a GEMV of n rows of k: enough warps to fill the device
    with whole rows where possible (one warp streams a row's split)."""
    for s in (1, 2, 4, 8):
        if (n_rows * s) >= sms * 48 or k // s < 1024:
            return s
    return 8


class Llama:
    """A Llama-shaped model on one device, or one rank of a Megatron-style
    tensor-parallel group: the weights (seeded on the device, or given), the
    Ring KV arena, the plans of the embedding, a layer and the head, and the
    captured decode step. Activations are f32; the weights and the caches
    are f32, bf16 or f16, as the shape says (`weights`, `cache`).

    With `world` ranks, each holds heads/world query and KV heads with their
    rows of q/k/v and columns of o, ffn/world rows of gate and up with their
    columns of down (column then row parallel), and vocab/world rows of the
    tied LM head; the embedding table is whole on every rank. The
    row-parallel projections (o, down) leave partial sums that an NCCL
    allreduce adds before their residual epilogue runs; the head's greedy
    candidates, one a shard, are gathered and picked.
    """

    def __init__(self, ctx: N.Context, shape: LlamaShape, batch: int, seed: int = 2026, chunk: int = 32,
                 pdl: bool = True, prefill_kv: float | None = None, rank: int = 0, world: int = 1,
                 host_weights=None, peer_exchange: bool = True, fuse_attention: bool | None = None,
                 selection: str | None = None, gated: bool = False, store_gelus: bool = False,
                 prefetch_attention: int = 0, prefetch_gemv: int | None = None):
        import dataclasses

        full = shape
        for what, n in (("heads", full.heads), ("kv_heads", full.kv_heads), ("ffn", full.ffn),
                        ("vocab", full.vocab)):
            if n % world:
                raise N.Refused(N.FKC_ERR_ARGUMENT, f"{what} {n} does not split over {world} ranks.")
        s = dataclasses.replace(full, heads=full.heads // world, kv_heads=full.kv_heads // world,
                                ffn=full.ffn // world)
        self.ctx, self.full, self.s, self.m = ctx, full, s, batch
        # The layer's plan options: a route in a step of its own (optGated),
        # gelus stored by their own step (optStoreGelus).
        self.gated, self.store_gelus = gated, store_gelus
        self.rank, self.world = rank, world
        # Bytes of a weight and of a cache element.
        self.wb = {"f32": 4, "bf16": 2, "f16": 2}.get(s.weights)
        self.cb = {"f32": 4, "bf16": 2, "f16": 2}.get(s.cache)
        if self.wb is None or self.cb is None:
            raise N.Refused(N.FKC_ERR_ARGUMENT, f"no kernels for {s.weights} weights and {s.cache} caches.")
        if s.experts > 1024:
            raise N.Refused(N.FKC_ERR_ARGUMENT, "routed experts: at most 1024 experts.")
        if s.experts and s.expert_scale and (s.experts * self.wb) % 16:
            raise N.Refused(N.FKC_ERR_ARGUMENT, "expert scales: the experts' scales must fill whole 16 bytes, so that "
                                                "the weights after them start on a 16-byte boundary.")
        if self.wb == 2 and any(n % 8 for n in (s.d_model, s.q_width, s.kv_width, s.ffn)):
            raise N.Refused(N.FKC_ERR_ARGUMENT, "16-bit weights: d_model, the q and kv widths and ffn must be "
                            "multiples of 8, so that every weight starts on a 16-byte boundary.")
        # For decode batches the streaming and batched GEMVs take (up to 64
        # rows), the arena interleaves gate and up rows (gate_i at row 2i, up_i at
        # 2i + 1), so that the [gate; up] step computes mlp_act = silu(gate) *
        # up on its own tiles and stores it, and the down step reads it: the
        # same bits as recomputing it in the down step, computed once.
        self.gate_up_interleaved = batch <= 64
        # Tensor parallelism's sums travel through peer memory (the context's
        # peer set, tp.init) for the batches the streaming GEMV takes; larger
        # batches use NCCL.
        # (Routed experts sum their ranks' shares by NCCL.)
        self.peer_exchange = world > 1 and batch <= 4 and peer_exchange and not s.experts
        self.vocab_local = full.vocab // world
        self.plans = {
            "embed": PL.plan(PL.DEFAULT, embed_program(full)),
            "layer": PL.plan(PL.PlanOptions(gated=gated, store_gelus=store_gelus,
                                            sequence_rows=batch if s.slots == 1 else 1), layer_program(s)),
            "head": PL.plan(PL.DEFAULT, head_program(dataclasses.replace(full, vocab=self.vocab_local))),
        }
        # Weights: per layer [q;k;v], o, [gate;up], down, two norms; then the
        # tied embedding/LM head and the final norm. N(0, 0.02), the norm
        # gains too (the configs give no other law for them).
        d, qw, kvw, f = s.d_model, s.q_width, s.kv_width, s.ffn
        self.layer_elems = sum(self.layer_sizes())
        wb = self.wb
        self.arena = ctx.alloc(wb * (s.layers * self.layer_elems + full.vocab * d + d))
        fill = self._fill(s.weights)
        if host_weights is None:
            # A rank's layer shards from its own seed; the embedding and the
            # norms alike on every rank (16-bit: the same values, rounded).
            layers = N.DeviceBuffer(ctx, self.arena.ptr, wb * s.layers * self.layer_elems)
            fill(layers, seed + 7919 * rank, 0.0, 0.02)
            rest = N.DeviceBuffer(ctx, self.embed_ptr(), wb * (full.vocab * d + d))
            fill(rest, seed + 104729, 0.0, 0.02)
            for l in range(s.layers):
                w = self.layer_weights(l)
                fill(N.DeviceBuffer(ctx, w["attn_norm"], 2 * wb * d), seed + 3 * l + 1, 0.0, 0.02)
                if s.experts:  # the router (and the experts' scales) whole on every rank
                    fill(N.DeviceBuffer(ctx, w["router"], wb * s.experts * d), seed + 611953 + l, 0.0, 0.02)
                    if s.expert_scale:
                        fill(N.DeviceBuffer(ctx, w["expert_scale"], wb * s.experts), seed + 711957 + l, 1.0, 0.25)
        else:
            self.arena.upload(host_weights)
        self.cos, self.sin = ctx.rope_tables(s.theta, s.head_dim, s.head_dim // 2, s.positions)
        self.kbase, self.vbase = self._kv_arena()
        if prefill_kv is not None:
            kv = s.layers * self._kv_units() * s.kv_heads * self._kv_unit_len() * s.head_dim
            cfill = self._fill(s.cache)
            cfill(N.DeviceBuffer(ctx, self.kbase, self.cb * kv), seed + 1 + 17 * rank, 0.0, prefill_kv)
            cfill(N.DeviceBuffer(ctx, self.vbase, self.cb * kv), seed + 2 + 17 * rank, 0.0, prefill_kv)
        m = batch
        # A step's row inputs in one buffer, so that one copy brings them in:
        # the tokens, the positions, the slots, each part on a 16-byte
        # boundary as every buffer a kernel binds (leastAlign,
        # src/FuryKernel/Type.hs:66-71).
        # With a paged cache the third part is the rows' block tables
        # [m, table_len] instead of their slots.
        self.row_stride = (m + 3) // 4 * 4
        seq = s.table_len if s.paged else 1
        self.rows_words = 2 * self.row_stride + (m * seq + 3) // 4 * 4
        self.rows = ctx.zeros(self.rows_words, np.uint32)
        rs = 4 * self.row_stride
        self.tokens = N.DeviceBuffer(ctx, self.rows.ptr, 4 * m, np.uint32, (m,))
        self.pos = N.DeviceBuffer(ctx, self.rows.ptr + rs, 4 * m, np.uint32, (m,))
        self.slot = N.DeviceBuffer(ctx, self.rows.ptr + 2 * rs, 4 * m * seq, np.uint32,
                                   (m, seq) if s.paged else (m,))
        self.out_ids = ctx.zeros(m, np.uint32)
        self.x = ctx.zeros((m, d))
        self.x1 = ctx.zeros((m, d))
        self.partial = ctx.zeros((m, d))
        self.qkv = ctx.zeros((m, qw + 2 * kvw))
        self.att = ctx.zeros((m, qw))
        self.gu = ctx.zeros((m, 2 * f))
        self.act = ctx.zeros((m, f))
        if s.experts:  # the routed FFN's rows: the normed row, logits, route, experts' in and out
            e, k = s.experts, s.top_k
            self.moe = {"mlp_in": ctx.zeros((m, d)), "router_logits": ctx.zeros((m, e)),
                        "route_ids": ctx.zeros((m, k), np.uint32), "route_weights": ctx.zeros((m, k)),
                        "experts_gu": ctx.zeros((m, k * 2 * f)), "experts_act": ctx.zeros((m, k * f)),
                        "experts_out": ctx.zeros((m, k * d))}
        self.logits = ctx.zeros((m, self.vocab_local))
        self.pairs = ctx.zeros(2 * m, np.uint32)
        self.pairs_all = ctx.zeros(2 * m * world, np.uint32)
        self.chunk = chunk
        self.max_splits = (s.positions + chunk - 1) // chunk
        self.part = [ctx.zeros(m * s.heads * self.max_splits), ctx.zeros(m * s.heads * self.max_splits),
                     ctx.zeros(m * s.heads * self.max_splits * s.head_dim)]
        self.pdl = pdl
        # The weight bytes each streaming GEMV brings toward L2 by bulk
        # prefetch before it waits for its predecessor (0: its first lines
        # only), and the next GEMV's weight bytes an attention launch brings
        # toward L2 while it runs. Measured on config 5 (same process,
        # repeated): 64 MiB a GEMV takes 2% off the batch-1 step and adds 2%
        # at batch 4, so it is the default at batch 1 only; the attention's
        # prefetch competes with its own KV loads and is off.
        self.prefetch_attention = prefetch_attention
        self.prefetch_gemv = (64 << 20 if batch == 1 else 0) if prefetch_gemv is None else prefetch_gemv
        # The decode step's KV store and attention as one launch
        # (attend_decode), for rows in distinct slots (set_rows checks): by
        # default for the small batches whose steps are launch-bound (one
        # launch a layer fewer); at batch 16 the separate store measured
        # faster (0.617 against 0.658 ms a layer at context 2048).
        # (No fused form reads a paged cache.)
        if fuse_attention is None:
            fuse_attention = m <= 4
        # (A paged cache's fused form needs every block-table entry
        # distinct: set_rows checks the tables it uploads.)
        self.fuse_attention = fuse_attention and m <= 64
        # A committed selection (furykernel_b200.select): each GEMV shape's
        # split-K, the same at every batch.
        self.splits = {}
        if selection is not None:
            from . import select

            self.splits = select.splits_for(self, selection)
        self.launches = self._launches()
        self.graph = None

    # -- layout
    def _kv_units(self) -> int:
        """A layer's ring slots, or its pool's blocks."""
        return self.s.blocks if self.s.paged else self.s.slots

    def _kv_unit_len(self) -> int:
        """Positions a slot or a block holds."""
        return self.s.block_size if self.s.paged else self.s.length

    def _kv_arena(self):
        import ctypes

        k, v = ctypes.c_void_p(), ctypes.c_void_p()
        s = self.s
        N.check(N.lib().fkc_kv_arena_elem(self.ctx.handle, s.layers, self._kv_units(), s.kv_heads,
                                          self._kv_unit_len(), s.head_dim, self.cb, ctypes.byref(k),
                                          ctypes.byref(v)))
        return k.value, v.value

    LAYER_ORDER = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj", "attn_norm",
                   "mlp_norm")
    # With routed experts: the router and the experts' tables (each entry
    # [2 ffn, d] gate/up and [d, ffn] down) in place of the dense FFN.
    MOE_ORDER = ("q_proj", "k_proj", "v_proj", "o_proj", "router", "experts_gate_up", "experts_down", "attn_norm",
                 "mlp_norm")

    def layer_order(self) -> tuple:
        if self.s.experts and getattr(self.s, "expert_scale", False):  # the scales after the router
            return self.MOE_ORDER[:5] + ("expert_scale",) + self.MOE_ORDER[5:]
        return self.MOE_ORDER if self.s.experts else self.LAYER_ORDER

    def _fill(self, t: str):
        """The seeded normal fill of elements of type t (16-bit: the f32
        fill's values, rounded)."""
        return {"f32": self.ctx.fill_normal, "bf16": self.ctx.fill_normal_bf16,
                "f16": self.ctx.fill_normal_f16}[t]

    def layer_sizes(self) -> list:
        s = self.s
        d, qw, kvw, f = s.d_model, s.q_width, s.kv_width, s.ffn
        if s.experts:
            scale = [s.experts] if getattr(s, "expert_scale", False) else []
            return [qw * d, kvw * d, kvw * d, d * qw, s.experts * d] + scale + \
                [s.experts * 2 * f * d, s.experts * d * f, d, d]
        return [qw * d, kvw * d, kvw * d, d * qw, f * d, f * d, d * f, d, d]

    def layer_weights(self, l: int) -> dict:
        base = self.arena.ptr + self.wb * l * self.layer_elems
        off, at = {}, 0
        for name, n in zip(self.layer_order(), self.layer_sizes()):
            off[name] = base + self.wb * at
            at += n
        return off

    def embed_ptr(self) -> int:
        return self.arena.ptr + self.wb * self.s.layers * self.layer_elems

    def final_norm_ptr(self) -> int:
        return self.embed_ptr() + self.wb * self.full.vocab * self.full.d_model

    def kv_layer(self, l: int):
        s = self.s
        per = self.cb * self._kv_units() * s.kv_heads * self._kv_unit_len() * s.head_dim
        return self.kbase + l * per, self.vbase + l * per

    # -- the step's launches
    def launch_addresses(self) -> dict:
        """The device addresses the decode step's launches bind (the C++
        host library's fkh_llama_desc)."""
        return {"arena": self.arena.ptr, "kbase": self.kbase, "vbase": self.vbase, "cos_t": self.cos.ptr,
                "sin_t": self.sin.ptr, "tokens": self.tokens.ptr, "pos": self.pos.ptr, "slot": self.slot.ptr,
                "x": self.x.ptr, "x1": self.x1.ptr, "qkv": self.qkv.ptr, "att": self.att.ptr, "gu": self.gu.ptr,
                "act": self.act.ptr, "logits": self.logits.ptr, "out_ids": self.out_ids.ptr,
                "partial": self.partial.ptr, "pairs": self.pairs.ptr, "pairs_all": self.pairs_all.ptr,
                "part": [b.ptr for b in self.part],
                **{name: buf.ptr for name, buf in getattr(self, "moe", {}).items()}}

    def _launches(self) -> list:
        """The decode step's launches, from libfurykernel_host.so
        (fkh_llama_launches): the plans of the embedding, a layer and the
        head lowered to table launches, then the rewrites below."""
        from . import _host

        return [Launch(k, p, b) for k, p, b in _host.llama_launches(*self.launch_args())]

    def launch_args(self) -> tuple:
        """fkh_llama_desc's fields: the shape, the batch, the rank, the
        choices and the addresses."""
        return (self.full, self.m, self.rank, self.world, self.ctx.sms, self.chunk, self.gate_up_interleaved,
                self.peer_exchange, self.fuse_attention, self.launch_addresses(), getattr(self, "splits", None),
                getattr(self, "gated", False), getattr(self, "store_gelus", False))

    def _launches_restated(self) -> list:
        """The same launch list in Python (the restatement the host
        library is checked against)."""
        s, m = self.s, self.m
        d, qw, kvw, f = s.d_model, s.q_width, s.kv_width, s.ffn
        tables = {"cos": self.cos.ptr, "sin": self.sin.ptr}
        ints = {"token": self.tokens.ptr, "position": self.pos.ptr,
                ("block_table" if s.paged else "slot"): self.slot.ptr}
        attn = {"chunk": self.chunk, "max_splits": self.max_splits, "partials": [b.ptr for b in self.part]}
        out = []
        eb = Binding(weights={"embed": self.embed_ptr()}, ints=ints, m=m, values={"x": View(self.x, 0, d, d)})
        p = self.plans["embed"].program
        for st in self.plans["embed"].steps:
            out.append(lower_step(p, st, eb, tables, attn))
        p = self.plans["layer"].program
        for l in range(s.layers):
            kc, vc = self.kv_layer(l)
            values = {"x": View(self.x, 0, d, d), "q": View(self.qkv, 0, qw + 2 * kvw, qw),
                      "k": View(self.qkv, qw, qw + 2 * kvw, kvw), "v": View(self.qkv, qw + kvw, qw + 2 * kvw, kvw),
                      "attended": View(self.att, 0, qw, qw), "x1": View(self.x1, 0, d, d),
                      "gate": View(self.gu, 0, 2 * f, f), "up": View(self.gu, f, 2 * f, f),
                      "x2": View(self.x, 0, d, d)}
            if s.experts:
                e, k = s.experts, s.top_k
                for name, width in (("mlp_in", d), ("router_logits", e), ("route_ids", k), ("route_weights", k),
                                    ("experts_gu", k * 2 * f), ("experts_act", k * f), ("experts_out", k * d)):
                    values[name] = View(self.moe[name], 0, width, width)
            b = Binding(weights=self.layer_weights(l), ints=ints, caches={"k_cache": kc, "v_cache": vc},
                        values=values, m=m)
            for st in self.plans["layer"].steps:
                out += lower_steps(p, st, b, tables, attn)
        p = self.plans["head"].program
        head_rows = self.embed_ptr() + self.wb * self.rank * self.vocab_local * d
        hb = Binding(weights={"embed": head_rows, "final_norm": self.final_norm_ptr()}, ints=ints, m=m,
                     values={"x": View(self.x, 0, d, d),
                             "logits": View(self.logits, 0, self.vocab_local, self.vocab_local),
                             "token": View(self.out_ids, 0, 1, 1)})
        for st in self.plans["head"].steps:
            out.append(lower_step(p, st, hb, tables, attn))
        if self.gate_up_interleaved:
            out = self._silu_on_tiles(out)
        if self.world > 1:
            out = self._tensor_parallel(out)
        if self.fuse_attention:
            out = self._fuse_attention(out)
        # The engine's greedy feedback: the ids become the next step's
        # tokens and the positions advance, so replays decode on their own.
        out.append(Launch("advance", {"m": m}, [self.out_ids.ptr, self.tokens.ptr, self.pos.ptr]))
        for L in out:  # split-K per GEMV shape (the routed GEMV keeps the lowering's split 1)
            if L.kernel.startswith("gemv") and not L.kernel.startswith("gemv_routed"):
                # A selection's pick for the shape, the same at every batch;
                # else one, which the streaming (m <= 4) and batched
                # (m <= 64) kernels keep (their parallelism is rows whatever
                # the split); past 64 rows the chunked kernel splits long rows.
                n, k = L.params["n"], L.params["k"]
                split = getattr(self, "splits", {}).get((n, k), 1 if m <= 64 else split_for(n, k, self.ctx.sms))
                if split != 1 and m > 4 and kernel_form(L.kernel)[0] in ("gemv_rmsnorm_silu",
                                                                         "gemv_reduce_rmsnorm_silu"):
                    raise N.Refused(N.FKC_ERR_ARGUMENT, f"{L.kernel}: the row-pair kernels take split 1 past batch 4, "
                                                        f"not {split}.")
                L.params["split"] = split
        return out

    def _fuse_attention(self, launches: list) -> list:
        """Each layer's KV store and split attention launches, when they bind
        the same row of q/k/v, positions, slots (or block tables) and caches,
        become one attend_decode (attend_decode_paged) launch (the same
        bits); the combine follows."""
        fused = {("kv_store_ring", "attend_split"): ("attend_decode", ("ldq", "rotated", "d", "kv_heads", "length")),
                 ("kv_store_paged", "attend_split_paged"): (
                     "attend_decode_paged", ("ldq", "rotated", "d", "kv_heads", "block_size", "table_len", "blocks"))}
        out, i = [], 0
        while i < len(launches):
            pair = [kernel_form(L.kernel) for L in launches[i:i + 2]]
            form = fused.get(tuple(b for b, _ in pair)) if i + 1 < len(launches) else None
            if form and pair[0][1] == pair[1][1]:
                kv, at = launches[i:i + 2]
                same = (kv.bufs[0] == at.bufs[0] and list(kv.bufs[3:7]) == list(at.bufs[3:7])
                        and all(kv.params[k] == at.params[k] for k in form[1]))
                if same:
                    p = dict(at.params, k_off=kv.params["k_off"], v_off=kv.params["v_off"])
                    out.append(Launch(form[0] + pair[0][1], p, list(at.bufs)))
                    i += 2
                    continue
            out.append(launches[i])
            i += 1
        return out

    def _silu_on_tiles(self, launches: list) -> list:
        """The [gate; up] step followed by the down step that recomputes
        silu(gate) * up from their stored rows becomes: the [gate; up] GEMV
        on interleaved rows with the SiLU-gate epilogue, storing mlp_act;
        the down GEMV reading it."""
        f = self.s.ffn
        gu = self.gu.ptr
        out = list(launches)
        for i in range(len(out) - 1):
            a, b = out[i], out[i + 1]
            (ab, asuf), (bb, bsuf) = kernel_form(a.kernel), kernel_form(b.kernel)
            if (ab == "gemv_rmsnorm" and a.bufs[3] == gu and a.params["n"] == 2 * f
                    and bb in ("gemv_silu", "gemv_silu_add") and b.bufs[1] == gu and b.params["up_off"] == f):
                out[i] = Launch("gemv_rmsnorm_silu" + asuf, dict(a.params, ldy=f),
                                [a.bufs[0], a.bufs[1], a.bufs[2], self.act.ptr])
                params = {k: v for k, v in b.params.items() if k != "up_off"}
                params["ldx"] = f
                if bb == "gemv_silu_add":
                    out[i + 1] = Launch("gemv_add" + bsuf, params, [b.bufs[0], self.act.ptr, b.bufs[2], b.bufs[3]])
                else:
                    out[i + 1] = Launch("gemv" + bsuf, params, [b.bufs[0], self.act.ptr, b.bufs[2]])
        return out

    def _tensor_parallel(self, launches: list) -> list:
        if self.peer_exchange and self.s.experts:
            raise Unlowerable(N.FKC_ERR_ARGUMENT, "routed experts over several ranks: their sums travel by NCCL, not "
                                                  "peer memory.")
        if self.peer_exchange:
            return self._tensor_parallel_peers(launches)
        return self._tensor_parallel_nccl(launches)

    def _tensor_parallel_peers(self, launches: list) -> list:
        """Over NVLink peer memory: a row-parallel projection scatters its
        partial rows into every rank's exchange buffer (o: 0, down: 1) and
        leaves its residual epilogue to the next GEMV, whose prologue adds
        the ranks' partials in rank order to the residual, stores the new
        residual row and normalizes it; the greedy candidates travel the
        same way. The same launches as on one GPU, no collective."""
        out, pending = [], None  # pending: (buffer, residual, where the sum goes)
        for L in launches:
            base, suf = kernel_form(L.kernel)
            if base == "gemv_add":
                w, x, r, y = L.bufs
                xbuf = 0 if pending is None or pending[0] == 1 else 1
                p = L.params
                if p["ldy"] != self.s.d_model or p["ldr"] != self.s.d_model:
                    raise Unlowerable(N.FKC_ERR_ARGUMENT, "a row-parallel output that is not a whole row.")
                out.append(Launch("gemv_scatter" + suf, {"n": p["n"], "k": p["k"], "m": p["m"], "split": p["split"],
                                                         "ldx": p["ldx"], "xbuf": xbuf}, [w, x]))
                pending = (xbuf, r, y)
            elif pending is not None and base in ("gemv_rmsnorm", "gemv_rmsnorm_silu") and L.bufs[1] == pending[2]:
                w, x, gamma, y = L.bufs
                p = dict(L.params)
                p.pop("ldx")
                p.update(ldr=self.s.d_model, xbuf=pending[0])
                name = "gemv_reduce_rmsnorm_silu" if base == "gemv_rmsnorm_silu" else "gemv_reduce_rmsnorm"
                out.append(Launch(name + suf, p, [w, pending[1], gamma, pending[2], y]))
                pending = (pending[0], None, None)  # consumed; the buffer alternates on
            elif L.kernel == "argmax":
                x, ids = L.bufs
                out.append(Launch("argmax_scatter", dict(L.params, offset=self.rank * self.vocab_local), [x]))
                out.append(Launch("argmax_gather_pick", {"m": self.m}, [ids]))
            else:
                out.append(L)
        return out

    def _tensor_parallel_nccl(self, launches: list) -> list:
        """With NCCL: the row-parallel projections' residual epilogues move
        after the allreduce of their partial sums, the experts' outputs (each
        rank's share of every expert's FFN) are summed before they are
        combined, and the greedy pick gathers the shards' candidates."""
        m, d = self.m, self.s.d_model
        P = self.partial.ptr
        out = []
        for L in launches:
            base, suf = kernel_form(L.kernel)
            if base in ("gemv_add", "gemv_silu_add"):
                w, x, r, y = L.bufs
                params = {k: v for k, v in L.params.items() if k != "ldr"}
                if params["ldy"] != d or L.params["ldr"] != d:
                    raise Unlowerable(N.FKC_ERR_ARGUMENT, "a row-parallel output that is not a whole row.")
                out.append(Launch(base[:-4] + suf, params, [w, x, P]))
                out.append(Launch("__allreduce__", {"count": m * d}, [P]))
                out.append(Launch("add", {"n": m * d}, [r, P, y]))
            elif L.kernel == "combine_ranks_add":
                p = L.params
                out.append(Launch("__allreduce__", {"count": p["m"] * p["k"] * p["d"]}, [L.bufs[2]]))
                out.append(L)
            elif L.kernel == "argmax":
                x, ids = L.bufs
                out.append(Launch("argmax_pairs", dict(L.params, offset=self.rank * self.vocab_local),
                                  [x, self.pairs.ptr]))
                out.append(Launch("__allgather__", {"count": 2 * m}, [self.pairs.ptr, self.pairs_all.ptr]))
                out.append(Launch("argmax_pick", {"shards": self.world, "m": m}, [self.pairs_all.ptr, ids]))
            else:
                out.append(L)
        return out

    def _run(self, L: Launch) -> None:
        if L.kernel == "__allreduce__":
            N.check(N.lib().fkc_allreduce_sum_f32(self.ctx.handle, L.bufs[0], L.params["count"]))
        elif L.kernel == "__allgather__":
            N.check(N.lib().fkc_allgather_u32(self.ctx.handle, L.bufs[0], L.bufs[1], L.params["count"]))
        else:
            L.run(self.ctx)

    ATTEND = ("attend_decode", "attend_split")

    def _next_gemv_weights(self, i: int):
        """(address, bytes) of the weights of the first GEMV after launch i."""
        for L in self.launches[i + 1:]:
            if L.kernel.startswith("gemv"):
                nbytes = self.wb * L.params["n"] * L.params["k"]
                return L.bufs[0], nbytes - nbytes % 16
        return 0, 0

    def _run_all(self) -> None:
        """The step's launches in order. Every streaming GEMV gets its own
        L2 prefetch budget (prefetch_gemv, fkc_set_prefetch); an attention
        launch brings the next GEMV's weights toward L2 while it runs (up to
        prefetch_attention bytes, fkc_set_l2_prefetch)."""
        if self.prefetch_gemv:
            self.ctx.set_prefetch(self.prefetch_gemv)
        try:
            for i, L in enumerate(self.launches):
                att = self.prefetch_attention > 0 and L.kernel.startswith(self.ATTEND)
                if att:
                    ptr, nbytes = self._next_gemv_weights(i)
                    self.ctx.set_l2_prefetch(ptr, min(nbytes, self.prefetch_attention))
                try:
                    self._run(L)
                finally:
                    if att:
                        self.ctx.set_l2_prefetch(0, 0)
        finally:
            if self.prefetch_gemv:
                self.ctx.set_prefetch(0)

    def run_eager(self) -> None:
        self.ctx.set_pdl(False)
        self._run_all()

    def capture(self) -> N.Graph:
        if self.graph is None:
            self.ctx.set_pdl(self.pdl)
            self.ctx.capture_begin()
            try:
                self._run_all()
            finally:
                g = self.ctx.capture_end()
                self.ctx.set_pdl(False)
            self.graph = g
        return self.graph

    def check_rows(self, tokens, positions, slots) -> None:
        """Refuses row inputs the kernels would index past their buffers
        with: ids past the vocabulary, positions past the RoPE tables, slots
        past the KV arena (or, paged, block-table entries past the pool)."""
        s = self.s
        seq = ("block", slots, s.blocks) if s.paged else ("slot", slots, s.slots)
        for what, v, bound in (("token", tokens, self.full.vocab), ("position", positions, s.positions), seq):
            v = np.asarray(v)
            if v.size and int(v.max()) >= bound:
                raise N.Refused(N.FKC_ERR_ARGUMENT, f"a {what} {int(v.max())} is past the engine's {bound}.")

    def set_rows(self, tokens, positions, slots=None) -> None:
        """A step's rows: tokens, positions, and each row's ring slot or,
        with a paged cache, its block table [m, table_len]."""
        if self.s.paged:
            if slots is None:
                raise N.Refused(N.FKC_ERR_ARGUMENT, "a paged cache's rows need their block tables.")
            slots = np.asarray(slots, np.uint32)
            if slots.shape != (self.m, self.s.table_len):
                raise N.Refused(N.FKC_ERR_ARGUMENT, f"block tables of shape {slots.shape}, not "
                                                    f"({self.m}, {self.s.table_len}).")
        slots = np.asarray(slots if slots is not None else np.arange(self.m), np.uint32)
        self.check_rows(tokens, positions, slots)
        if self.fuse_attention and np.unique(slots).size != slots.size:
            what = "every block-table entry distinct" if self.s.paged else "its rows in distinct slots"
            raise N.Refused(N.FKC_ERR_ARGUMENT, f"a decode step needs {what} (the fused attention stores a row's "
                                                "key while the others read).")
        self.tokens.upload(np.asarray(tokens, np.uint32))
        self.pos.upload(np.asarray(positions, np.uint32))
        self.slot.upload(slots)

    def step(self) -> np.ndarray:
        self.capture().launch()
        self.ctx.sync()
        return self.out_ids.download()

    def launch_count(self) -> int:
        """Kernels of this library a step launches (collectives excluded)."""
        return sum(1 for L in self.launches if not L.kernel.startswith("__"))

    def weight_bytes(self) -> int:
        """The weights a step streams on this rank: the layers' shards, the
        LM head's vocabulary rows and the final norm."""
        s = self.s
        return self.wb * (s.layers * self.layer_elems + self.vocab_local * s.d_model + s.d_model)

    def algorithmic_bytes(self, contexts) -> int:
        """Bytes a decode step must move on this rank: every weight once, each
        row's keys and values over its context, per layer."""
        s = self.s
        kv = sum(2 * s.kv_heads * s.head_dim * self.cb * (int(c) + 1) for c in contexts) * s.layers
        return self.weight_bytes() + kv


def shard_weights(full: LlamaShape, layers: list, embed: np.ndarray, final_norm: np.ndarray, rank: int,
                  world: int, interleave: bool = False) -> np.ndarray:
    """One rank's weight arena from the whole model's host weights, in the
    engine's layout: per layer q/k/v rows of its heads, o's columns of its
    heads, gate/up rows of its ffn slice, down's columns of that slice,
    the norms; then the whole embedding and the final norm.

    `layers` holds per layer the f32 arrays q [H*hd, d], k and v
    [KV*hd, d], o [d, H*hd], gate and up [F, d], down [d, F], attn_norm and
    mlp_norm [d]; with routed experts, router [E, d], expert_scale [E] (with
    the shape's expert_scale), egu [E, 2F, d] (each expert's gate rows, then
    its up rows) and edn [E, d, F] in place of gate, up and down. A rank
    holds the whole router and scales and, of every expert, the gate and up
    rows and the down columns of its ffn slice."""
    hd, d = full.head_dim, full.d_model
    hq, hk, fl = full.heads // world, full.kv_heads // world, full.ffn // world
    qs = slice(rank * hq * hd, (rank + 1) * hq * hd)
    ks = slice(rank * hk * hd, (rank + 1) * hk * hd)
    fs = slice(rank * fl, (rank + 1) * fl)
    parts = []
    for w in layers:
        parts += [w["q"][qs], w["k"][ks], w["v"][ks], np.ascontiguousarray(w["o"][:, qs])]
        if full.experts:
            f = full.ffn
            egu = np.concatenate([w["egu"][:, fs], w["egu"][:, f + rank * fl:f + (rank + 1) * fl]], axis=1)
            parts += [w["router"]] + ([w["expert_scale"]] if full.expert_scale else [])
            parts += [egu, np.ascontiguousarray(w["edn"][:, :, fs]), w["attn_norm"], w["mlp_norm"]]
            continue
        gate, up = w["gate"][fs], w["up"][fs]
        gu = np.stack([gate, up], axis=1).reshape(2 * fl, d) if interleave else [gate, up]
        parts += [gu] if interleave else gu
        parts += [np.ascontiguousarray(w["down"][:, fs]), w["attn_norm"], w["mlp_norm"]]
    parts += [embed, final_norm]
    return np.concatenate([np.ascontiguousarray(a, np.float32).ravel() for a in parts])
