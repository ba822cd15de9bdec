"""ctypes binding of libfurykernel_host.so (include/furykernel_host.h): the
programs, the planner and the lowering in C++. The Llama engine takes its
launch list from here; the Python restatement under `tests/restated/` is the
same algorithm, kept as the checker the tests compare against."""

from __future__ import annotations

import ctypes
import os

from . import _native as N

_LIB = None
_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_build", "libfurykernel_host.so")

FKH_OK, FKH_ERR_ARGUMENT, FKH_ERR_SPACE, FKH_ERR_INTERNAL = 0, 1, 2, 3
ABI_VERSION = 9


# The shape's element-type codes, in order (fkh_llama_shape).
ELEMENT_TYPES = ("f32", "bf16", "f16")


class Shape(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint64) for n in ("d_model", "heads", "kv_heads", "head_dim", "ffn", "vocab",
                                                "layers")] + \
               [("theta", ctypes.c_double), ("eps", ctypes.c_double)] + \
               [(n, ctypes.c_uint64) for n in ("slots", "length", "positions")] + \
               [("weights_type", ctypes.c_int), ("cache_type", ctypes.c_int)] + \
               [("blocks", ctypes.c_uint64), ("block_size", ctypes.c_uint64)] + \
               [("experts", ctypes.c_uint64), ("top_k", ctypes.c_uint64)] + \
               [("expert_scale", ctypes.c_int)]


class PlanOptions(ctypes.Structure):
    _fields_ = [("horizontal", ctypes.c_int), ("gated", ctypes.c_int), ("store_gelus", ctypes.c_int),
                ("sequence_rows", ctypes.c_uint64)]


DESC_ADDRS = ("arena", "kbase", "vbase", "cos_t", "sin_t", "tokens", "pos", "slot", "x", "x1", "qkv", "att", "gu",
              "act", "logits", "out_ids", "partial", "pairs", "pairs_all")


MOE_ADDRS = ("mlp_in", "router_logits", "route_ids", "route_weights", "experts_gu", "experts_act", "experts_out")


class Desc(ctypes.Structure):
    _fields_ = [("full", Shape)] + \
               [(n, ctypes.c_uint64) for n in ("batch", "rank", "world", "sms", "chunk")] + \
               [(n, ctypes.c_int) for n in ("gate_up_interleaved", "peer_exchange", "fuse_attention")] + \
               [(n, ctypes.c_uint64) for n in DESC_ADDRS] + [("part", ctypes.c_uint64 * 3)] + \
               [("splits", ctypes.POINTER(ctypes.c_uint32)), ("nsplits", ctypes.c_size_t)] + \
               [(n, ctypes.c_uint64) for n in MOE_ADDRS] + \
               [("gated", ctypes.c_int), ("store_gelus", ctypes.c_int)]


def lib():
    """The loaded library, rebuilt first (g++, no CUDA) when a source is
    newer; a failed build or load raises."""
    global _LIB
    if _LIB is None:
        from . import build as B

        B.build_host()  # a no-op unless a source is newer than the library
        L = ctypes.CDLL(_PATH)
        L.fkh_abi_version.restype = ctypes.c_int
        if L.fkh_abi_version() != ABI_VERSION:
            raise RuntimeError(f"libfurykernel_host.so has ABI {L.fkh_abi_version()}, this binding {ABI_VERSION}")
        text_args = [ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t), ctypes.c_char_p,
                     ctypes.c_size_t]
        L.fkh_llama_program_text.argtypes = [ctypes.POINTER(Shape), ctypes.c_int] + text_args
        L.fkh_program_roundtrip.argtypes = [ctypes.c_char_p] + text_args
        L.fkh_plan_text.argtypes = [ctypes.c_char_p, ctypes.POINTER(PlanOptions)] + text_args
        L.fkh_llama_launches.argtypes = [ctypes.POINTER(Desc), ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p,
                                         ctypes.c_size_t]
        L.fkh_llama_prefill_launches.argtypes = [ctypes.POINTER(Desc), ctypes.POINTER(PrefillDesc), ctypes.c_uint64,
                                                 ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p, ctypes.c_size_t]
        L.fkh_launches_count.argtypes = [ctypes.c_void_p]
        L.fkh_launches_count.restype = ctypes.c_size_t
        for f in ("fkh_launch_param_count", "fkh_launch_buf_count"):
            getattr(L, f).argtypes = [ctypes.c_void_p, ctypes.c_size_t]
            getattr(L, f).restype = ctypes.c_size_t
        L.fkh_launch_kernel.argtypes = [ctypes.c_void_p, ctypes.c_size_t]
        L.fkh_launch_kernel.restype = ctypes.c_char_p
        L.fkh_launch_param_name.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t]
        L.fkh_launch_param_name.restype = ctypes.c_char_p
        L.fkh_launch_param_value.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t]
        L.fkh_launch_param_value.restype = ctypes.c_double
        L.fkh_launch_buf.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t]
        L.fkh_launch_buf.restype = ctypes.c_uint64
        L.fkh_launches_free.argtypes = [ctypes.c_void_p]
        L.fkh_split_for.argtypes = [ctypes.c_uint64] * 3
        L.fkh_split_for.restype = ctypes.c_uint64
        _LIB = L
    return _LIB


def _check(rc: int, err) -> None:
    if rc == FKH_ERR_ARGUMENT:
        raise N.Refused(N.FKC_ERR_ARGUMENT, err.value.decode())
    if rc != FKH_OK:
        raise N.FkcError(N.FKC_ERR_STATE, f"libfurykernel_host.so: {err.value.decode()} (code {rc})")


def _text(call, *args) -> str:
    err = ctypes.create_string_buffer(1024)
    n = ctypes.c_size_t(0)
    rc = call(*args, None, 0, ctypes.byref(n), err, len(err))
    if rc != FKH_ERR_SPACE:
        _check(rc, err)
    buf = ctypes.create_string_buffer(n.value + 1)
    _check(call(*args, buf, len(buf), ctypes.byref(n), err, len(err)), err)
    return buf.value.decode()


def shape(s) -> Shape:
    """A LlamaShape (furykernel_b200.shape) as the C struct."""
    for what, t in (("weights", s.weights), ("cache", s.cache)):
        if t not in ELEMENT_TYPES:
            raise N.Refused(N.FKC_ERR_ARGUMENT, f"the {what}' element type {t} is not f32, bf16 or f16.")
    return Shape(s.d_model, s.heads, s.kv_heads, s.head_dim, s.ffn, s.vocab, s.layers, s.theta, s.eps, s.slots,
                 s.length, s.positions, ELEMENT_TYPES.index(s.weights), ELEMENT_TYPES.index(s.cache), s.blocks,
                 s.block_size, s.experts, s.top_k, int(getattr(s, "expert_scale", False)))


def llama_program_text(s, which: str) -> str:
    """The rendered embed, layer or head program of a LlamaShape."""
    w = {"embed": 0, "layer": 1, "head": 2}[which]
    sh = shape(s)
    return _text(lib().fkh_llama_program_text, ctypes.byref(sh), w)


def program_roundtrip(text: str) -> str:
    return _text(lib().fkh_program_roundtrip, text.encode())


def plan_text(program_text: str, horizontal=True, gated=False, store_gelus=False, sequence_rows=1) -> str:
    """Plans a rendered program and renders the plan."""
    o = PlanOptions(int(horizontal), int(gated), int(store_gelus), sequence_rows)
    return _text(lib().fkh_plan_text, program_text.encode(), ctypes.byref(o))


def split_for(n_rows: int, k: int, sms: int) -> int:
    return int(lib().fkh_split_for(n_rows, k, sms))


def _desc(full, batch, rank, world, sms, chunk, gate_up_interleaved, peer_exchange, fuse_attention, addrs,
          splits=None, gated=False, store_gelus=False) -> Desc:
    """The descriptor; `splits` maps GEMV shapes (n, k) to a selection's
    split-K (the array stays alive as the descriptor's `_keep`); `gated`
    and `store_gelus` are the layer's plan options."""
    d = Desc()
    d.gated, d.store_gelus = int(gated), int(store_gelus)
    if splits:
        flat = (ctypes.c_uint32 * (3 * len(splits)))(*[v for (n, k), s in sorted(splits.items()) for v in (n, k, s)])
        d.splits, d.nsplits = ctypes.cast(flat, ctypes.POINTER(ctypes.c_uint32)), len(splits)
        d._keep = flat
    d.full = shape(full)
    d.batch, d.rank, d.world, d.sms, d.chunk = batch, rank, world, sms, chunk
    d.gate_up_interleaved, d.peer_exchange, d.fuse_attention = (int(gate_up_interleaved), int(peer_exchange),
                                                                 int(fuse_attention))
    for n in DESC_ADDRS + MOE_ADDRS:
        setattr(d, n, int(addrs.get(n, 0)))
    for i, p in enumerate(addrs["part"]):
        d.part[i] = int(p)
    return d


def _collect(call, *args) -> list:
    """A launch list from an entry that makes one: (kernel, params dict,
    bufs list) triples, params as ints where they are integers."""
    L = lib()
    h = ctypes.c_void_p()
    err = ctypes.create_string_buffer(1024)
    _check(call(*args, ctypes.byref(h), err, len(err)), err)
    try:
        out = []
        for i in range(L.fkh_launches_count(h)):
            params = {}
            for j in range(L.fkh_launch_param_count(h, i)):
                v = L.fkh_launch_param_value(h, i, j)
                params[L.fkh_launch_param_name(h, i, j).decode()] = int(v) if float(v).is_integer() else v
            bufs = [int(L.fkh_launch_buf(h, i, j)) for j in range(L.fkh_launch_buf_count(h, i))]
            out.append((L.fkh_launch_kernel(h, i).decode(), params, bufs))
        return out
    finally:
        L.fkh_launches_free(h)


def llama_launches(full, batch: int, rank: int, world: int, sms: int, chunk: int, gate_up_interleaved: bool,
                   peer_exchange: bool, fuse_attention: bool, addrs: dict, splits=None, gated=False,
                   store_gelus=False) -> list:
    """The decode step's launch list (fkh_llama_launches)."""
    d = _desc(full, batch, rank, world, sms, chunk, gate_up_interleaved, peer_exchange, fuse_attention, addrs,
              splits, gated, store_gelus)
    return _collect(lib().fkh_llama_launches, ctypes.byref(d))


PREFILL_ADDRS = ("w_hi", "w_lo", "tokens", "pos", "slot", "x", "a", "a_hi", "a_lo", "qkv", "att", "tmp", "x1",
                 "gu", "act")


PREFILL_MOE_ADDRS = ("router_logits", "route_ids", "route_weights", "experts_gu", "experts_act", "experts_out")


class PrefillDesc(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint64) for n in ("rows", "chunk", "positions")] + [("one_slot", ctypes.c_int)] + \
               [(n, ctypes.c_uint64) for n in PREFILL_ADDRS] + [("part", ctypes.c_uint64 * 3)] + \
               [(n, ctypes.c_uint64) for n in PREFILL_MOE_ADDRS]


def prefill_launches(decode: tuple, rows: int, chunk: int, positions: int, one_slot: bool, addrs: dict,
                     m: int) -> list:
    """The prefill of m rows (fkh_llama_prefill_launches); `decode` holds
    llama_launches' arguments for the engine in front of it."""
    d = _desc(*decode)
    p = PrefillDesc()
    p.rows, p.chunk, p.positions, p.one_slot = rows, chunk, positions, int(one_slot)
    for n in PREFILL_ADDRS:
        setattr(p, n, int(addrs[n]))
    for n in PREFILL_MOE_ADDRS:
        setattr(p, n, int(addrs.get(n, 0)))
    for i, a in enumerate(addrs["part"]):
        p.part[i] = int(a)
    return _collect(lib().fkh_llama_prefill_launches, ctypes.byref(d), ctypes.byref(p), m)


# ---- variant spaces and selections -----------------------------------------

def _setup_select(L):
    text = [ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t), ctypes.c_char_p, ctypes.c_size_t]
    L.fkh_json_roundtrip.argtypes = [ctypes.c_char_p] + text
    L.fkh_selection_roundtrip.argtypes = [ctypes.c_char_p] + text
    L.fkh_space_check.argtypes = [ctypes.c_char_p] + text
    L.fkh_space_parse_key.argtypes = [ctypes.c_char_p, ctypes.c_char_p] + text
    L.fkh_space_names.argtypes = [ctypes.c_char_p] + text
    L.fkh_split_join.argtypes = [ctypes.c_char_p, ctypes.c_char_p] + text
    u32p = ctypes.POINTER(ctypes.c_uint32)
    L.fkh_gemv_consider.argtypes = [ctypes.c_uint32] * 5 + [ctypes.POINTER(ctypes.c_int),
                                                           ctypes.POINTER(ctypes.c_uint64),
                                                           ctypes.POINTER(ctypes.c_uint64), ctypes.c_char_p,
                                                           ctypes.c_size_t]
    L.fkh_gemv_selection_render.argtypes = [u32p, u32p, ctypes.c_size_t, ctypes.c_uint32] + text
    L.fkh_gemv_selection_validate.argtypes = [ctypes.c_char_p, u32p, ctypes.c_size_t, ctypes.c_uint32, u32p,
                                              ctypes.c_char_p, ctypes.c_size_t]


def _lib_select():
    L = lib()
    if not getattr(L, "_select_ready", False):
        _setup_select(L)
        L._select_ready = True
    return L


def json_roundtrip(text: str) -> str:
    """JSON parsed and rendered as the reference renders it."""
    return _text(_lib_select().fkh_json_roundtrip, text.encode())


def selection_roundtrip(text: str) -> str:
    """A selection's JSON parsed and rendered back (the format only)."""
    return _text(_lib_select().fkh_selection_roundtrip, text.encode())


def space_check(space_json: str) -> list:
    """What checkSpace refuses of a space given as JSON."""
    out = _text(_lib_select().fkh_space_check, space_json.encode())
    return [p for p in out.split("\n") if p]


def space_parse_key(space_json: str, key: str) -> str:
    return _text(_lib_select().fkh_space_parse_key, space_json.encode(), key.encode())


def space_names(space_json: str) -> list:
    return [n for n in _text(_lib_select().fkh_space_names, space_json.encode()).split("\n") if n]


def split_join(name: str, right_prefix: str):
    out = _text(_lib_select().fkh_split_join, name.encode(), right_prefix.encode())
    return tuple(out.split("\n")) if out else None


GEMV_OUTCOMES = ("kept", "illegal", "indivisible", "too few")


def gemv_consider(n: int, k: int, m: int, split: int, cores: int) -> tuple:
    """What pruning makes of GEMV variant s<split> of class n_k_m:
    (outcome, work units, kernel identity, reasons)."""
    kind, groups, h = ctypes.c_int(), ctypes.c_uint64(), ctypes.c_uint64()
    reasons = ctypes.create_string_buffer(512)
    _check(_lib_select().fkh_gemv_consider(n, k, m, split, cores, ctypes.byref(kind), ctypes.byref(groups),
                                           ctypes.byref(h), reasons, len(reasons)), reasons)
    return GEMV_OUTCOMES[kind.value], groups.value, h.value, reasons.value.decode()


def _classes(classes):
    flat = (ctypes.c_uint32 * (3 * len(classes)))(*[int(v) for c in classes for v in c])
    return flat, len(classes)


def gemv_selection_render(classes, splits, cores: int) -> str:
    """A selection of this target's GEMV family: classes (n, k, m), each
    its split."""
    flat, n = _classes(classes)
    sp = (ctypes.c_uint32 * n)(*splits)
    return _text(_lib_select().fkh_gemv_selection_render, flat, sp, n, cores)


def gemv_selection_validate(text: str, classes, cores: int) -> list:
    """Each class's split from a committed selection, or a Refused with
    every problem, one a line."""
    flat, n = _classes(classes)
    out = (ctypes.c_uint32 * max(n, 1))()
    err = ctypes.create_string_buffer(8192)
    _check(_lib_select().fkh_gemv_selection_validate(text.encode(), flat, n, cores, out, err, len(err)), err)
    return list(out[:n])
