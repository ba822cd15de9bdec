"""Test infrastructure: the Python restatement of the host library's
lowering (libfurykernel_host.so, fkh_llama_launches): a plan's steps
(src/FuryKernel/Program/Plan.hs:109-121) become one launch each of a kernel
in the target's table -- the step's anchors set the kernel, its recomputed
operations become the kernel's prologue and its epilogues the kernel's
epilogue -- then the engine's rewrites (the SiLU-gate on interleaved
gate/up tiles, tensor parallelism over peer memory or NCCL, the fused
decode attention) and the split-K choice. The tests hold the C++ library
to it launch for launch; nothing in the package imports it.

Memory: a stored value lives in a device buffer of its rows; the anchors of
one step (horizontal q/k/v, gate/up) write adjacent columns of one buffer,
and their weights lie adjacent in the weight arena, so the step is one GEMV
over the concatenated rows."""

from __future__ import annotations

import dataclasses
from dataclasses import dataclass, field

from furykernel_b200 import _native as N
from furykernel_b200.engine import Launch, kernel_form
from furykernel_b200.target import CACHE_SUFFIX, WEIGHT_SUFFIX

from . import plan as PL
from .graph import Paged
from .llama import embed_program, head_program, layer_program


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
class Binding:
    """What a program's sources and stored values are on the device."""

    weights: dict = field(default_factory=dict)  # source name -> address
    ints: dict = field(default_factory=dict)  # source name -> address of [m] u32
    caches: dict = field(default_factory=dict)  # source name -> address of the layer's Ring
    values: dict = field(default_factory=dict)  # value name -> View
    m: int = 1


def _work_text(p, step) -> str:
    return "; ".join(f"{w.kind.lower()} {p.node(w.node).name}" for w in step.work)


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
                           part[0], part[1], part[2], b.caches[kc], b.caches[vc]])  # the tables after the buffers
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


def decode_plans(eng) -> dict:
    """The plans of an engine's embedding, layer and head (with the layer's
    plan options), as the host library plans them."""
    s, full = eng.s, eng.full
    return {
        "embed": PL.plan(PL.DEFAULT, embed_program(full)),
        "layer": PL.plan(PL.PlanOptions(gated=eng.gated, store_gelus=eng.store_gelus,
                                        sequence_rows=eng.m if s.slots == 1 else 1), layer_program(s)),
        "head": PL.plan(PL.DEFAULT, head_program(dataclasses.replace(full, vocab=eng.vocab_local))),
    }


def decode_launches(eng) -> list:
    """An engine's decode-step launch list in Python: the restatement the
    host library's fkh_llama_launches is checked against."""
    plans = decode_plans(eng)
    s, m = eng.s, eng.m
    d, qw, kvw, f = s.d_model, s.q_width, s.kv_width, s.ffn
    tables = {"cos": eng.cos.ptr, "sin": eng.sin.ptr}
    ints = {"token": eng.tokens.ptr, "position": eng.pos.ptr,
            ("block_table" if s.paged else "slot"): eng.slot.ptr}
    attn = {"chunk": eng.chunk, "max_splits": eng.max_splits, "partials": [b.ptr for b in eng.part]}
    out = []
    eb = Binding(weights={"embed": eng.embed_ptr()}, ints=ints, m=m, values={"x": View(eng.x, 0, d, d)})
    p = plans["embed"].program
    for st in plans["embed"].steps:
        out.append(lower_step(p, st, eb, tables, attn))
    p = plans["layer"].program
    for l in range(s.layers):
        kc, vc = eng.kv_layer(l)
        values = {"x": View(eng.x, 0, d, d), "q": View(eng.qkv, 0, qw + 2 * kvw, qw),
                  "k": View(eng.qkv, qw, qw + 2 * kvw, kvw), "v": View(eng.qkv, qw + kvw, qw + 2 * kvw, kvw),
                  "attended": View(eng.att, 0, qw, qw), "x1": View(eng.x1, 0, d, d),
                  "gate": View(eng.gu, 0, 2 * f, f), "up": View(eng.gu, f, 2 * f, f),
                  "x2": View(eng.x, 0, d, d)}
        if s.experts:
            e, k = s.experts, s.top_k
            for name, width in (("mlp_in", d), ("router_logits", e), ("route_ids", k), ("route_weights", k),
                                ("experts_gu", k * 2 * f), ("experts_act", k * f), ("experts_out", k * d)):
                values[name] = View(eng.moe[name], 0, width, width)
        b = Binding(weights=eng.layer_weights(l), ints=ints, caches={"k_cache": kc, "v_cache": vc},
                    values=values, m=m)
        for st in plans["layer"].steps:
            out += lower_steps(p, st, b, tables, attn)
    p = plans["head"].program
    head_rows = eng.embed_ptr() + eng.wb * eng.rank * eng.vocab_local * d
    hb = Binding(weights={"embed": head_rows, "final_norm": eng.final_norm_ptr()}, ints=ints, m=m,
                 values={"x": View(eng.x, 0, d, d),
                         "logits": View(eng.logits, 0, eng.vocab_local, eng.vocab_local),
                         "token": View(eng.out_ids, 0, 1, 1)})
    for st in plans["head"].steps:
        out.append(lower_step(p, st, hb, tables, attn))
    if eng.gate_up_interleaved:
        out = silu_on_tiles(eng, out)
    if eng.world > 1:
        out = tensor_parallel(eng, out)
    if eng.fuse_attention:
        out = fuse_attention(eng, out)
    # The engine's greedy feedback: the ids become the next step's
    # tokens and the positions advance, so replays decode on their own.
    out.append(Launch("advance", {"m": m}, [eng.out_ids.ptr, eng.tokens.ptr, eng.pos.ptr]))
    for L in out:  # split-K per GEMV shape (the routed GEMV keeps the lowering's split 1)
        if L.kernel.startswith("gemv") and not L.kernel.startswith("gemv_routed"):
            # A selection's pick for the shape, the same at every batch;
            # else one, which the streaming (m <= 4) and batched
            # (m <= 64) kernels keep (their parallelism is rows whatever
            # the split); past 64 rows the chunked kernel splits long rows.
            n, k = L.params["n"], L.params["k"]
            split = getattr(eng, "splits", {}).get((n, k), 1 if m <= 64 else split_for(n, k, eng.ctx.sms))
            if split != 1 and m > 4 and kernel_form(L.kernel)[0] in ("gemv_rmsnorm_silu",
                                                                     "gemv_reduce_rmsnorm_silu"):
                raise N.Refused(N.FKC_ERR_ARGUMENT, f"{L.kernel}: the row-pair kernels take split 1 past batch 4, "
                                                    f"not {split}.")
            L.params["split"] = split
    return out

def fuse_attention(eng, launches: list) -> list:
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
            tabs = 5 if pair[1][0] == "attend_split" else 8  # a ring's cache buffers, or a paged cache's tables
            same = (kv.bufs[0] == at.bufs[0] and list(kv.bufs[3:5]) == list(at.bufs[3:5])
                    and list(kv.bufs[5:7]) == list(at.bufs[tabs:tabs + 2])
                    and all(kv.params[k] == at.params[k] for k in form[1]))
            if same:
                p = dict(at.params, k_off=kv.params["k_off"], v_off=kv.params["v_off"])
                out.append(Launch(form[0] + pair[0][1], p, list(at.bufs)))
                i += 2
                continue
        out.append(launches[i])
        i += 1
    return out

def silu_on_tiles(eng, launches: list) -> list:
    """The [gate; up] step followed by the down step that recomputes
    silu(gate) * up from their stored rows becomes: the [gate; up] GEMV
    on interleaved rows with the SiLU-gate epilogue, storing mlp_act;
    the down GEMV reading it."""
    f = eng.s.ffn
    gu = eng.gu.ptr
    out = list(launches)
    for i in range(len(out) - 1):
        a, b = out[i], out[i + 1]
        (ab, asuf), (bb, bsuf) = kernel_form(a.kernel), kernel_form(b.kernel)
        if (ab == "gemv_rmsnorm" and a.bufs[3] == gu and a.params["n"] == 2 * f
                and bb in ("gemv_silu", "gemv_silu_add") and b.bufs[1] == gu and b.params["up_off"] == f):
            out[i] = Launch("gemv_rmsnorm_silu" + asuf, dict(a.params, ldy=f),
                            [a.bufs[0], a.bufs[1], a.bufs[2], eng.act.ptr])
            params = {k: v for k, v in b.params.items() if k != "up_off"}
            params["ldx"] = f
            if bb == "gemv_silu_add":
                out[i + 1] = Launch("gemv_add" + bsuf, params, [b.bufs[0], eng.act.ptr, b.bufs[2], b.bufs[3]])
            else:
                out[i + 1] = Launch("gemv" + bsuf, params, [b.bufs[0], eng.act.ptr, b.bufs[2]])
    return out

def tensor_parallel(eng, launches: list) -> list:
    if eng.peer_exchange and eng.s.experts:
        raise Unlowerable(N.FKC_ERR_ARGUMENT, "routed experts over several ranks: their sums travel by NCCL, not "
                                              "peer memory.")
    if eng.peer_exchange:
        return tensor_parallel_peers(eng, launches)
    return tensor_parallel_nccl(eng, launches)

def tensor_parallel_peers(eng, launches: list) -> list:
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
            if p["ldy"] != eng.s.d_model or p["ldr"] != eng.s.d_model:
                raise Unlowerable(N.FKC_ERR_ARGUMENT, "a row-parallel output that is not a whole row.")
            out.append(Launch("gemv_scatter" + suf, {"n": p["n"], "k": p["k"], "m": p["m"], "split": p["split"],
                                                     "ldx": p["ldx"], "xbuf": xbuf}, [w, x]))
            pending = (xbuf, r, y)
        elif pending is not None and base in ("gemv_rmsnorm", "gemv_rmsnorm_silu") and L.bufs[1] == pending[2]:
            w, x, gamma, y = L.bufs
            p = dict(L.params)
            p.pop("ldx")
            p.update(ldr=eng.s.d_model, xbuf=pending[0])
            name = "gemv_reduce_rmsnorm_silu" if base == "gemv_rmsnorm_silu" else "gemv_reduce_rmsnorm"
            out.append(Launch(name + suf, p, [w, pending[1], gamma, pending[2], y]))
            pending = (pending[0], None, None)  # consumed; the buffer alternates on
        elif L.kernel == "argmax":
            x, ids = L.bufs
            out.append(Launch("argmax_scatter", dict(L.params, offset=eng.rank * eng.vocab_local), [x]))
            out.append(Launch("argmax_gather_pick", {"m": eng.m}, [ids]))
        else:
            out.append(L)
    return out

def tensor_parallel_nccl(eng, launches: list) -> list:
    """With NCCL: the row-parallel projections' residual epilogues move
    after the allreduce of their partial sums, the experts' outputs (each
    rank's share of every expert's FFN) are summed before they are
    combined, and the greedy pick gathers the shards' candidates."""
    m, d = eng.m, eng.s.d_model
    P = eng.partial.ptr
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
            out.append(Launch("argmax_pairs", dict(L.params, offset=eng.rank * eng.vocab_local),
                              [x, eng.pairs.ptr]))
            out.append(Launch("__allgather__", {"count": 2 * m}, [eng.pairs.ptr, eng.pairs_all.ptr]))
            out.append(Launch("argmax_pick", {"shards": eng.world, "m": m}, [eng.pairs_all.ptr, ids]))
        else:
            out.append(L)
    return out
