"""The C++ host library (libfurykernel_host.so, include/furykernel_host.h)
against the Python restatement of the same programs, planner and lowering,
on the CPU: the rendered programs, the plans of the reference's golden
programs (test/Test/FuryKernel/ProgramTest.hs) under every option set, and
the Llama engine's whole decode-step launch list for every configuration
the tests and the bench run (addresses are stand-ins; nothing runs)."""

import ctypes
import dataclasses
import math
from types import SimpleNamespace

import numpy as np
import pytest

from furykernel_b200 import _host as H
from furykernel_b200 import _native as N
from furykernel_b200.engine import Llama
from furykernel_b200.shape import LlamaShape
from tests.restated import lowering as RL
from tests.restated import plan as PL
from tests.restated import prefill as RP
from tests.restated.build import program
from tests.restated.graph import render_program, whole_row
from tests.restated.llama import embed_program, head_program, layer_program

from tests.test_program import LAYER_PLAN, OPTION_SETS, two_tiles
from tests.test_program import head_program as golden_head
from tests.test_program import layer as golden_layer

SHAPES = [
    LlamaShape(),
    LlamaShape(d_model=512, heads=4, kv_heads=4, head_dim=128, ffn=1024, vocab=3000, layers=2, slots=3, length=96,
               positions=96),
    LlamaShape(d_model=64, heads=4, kv_heads=2, head_dim=8, ffn=48, vocab=40, layers=2, slots=1, length=16,
               positions=16),
    LlamaShape(d_model=128, heads=8, kv_heads=8, head_dim=16, ffn=344, vocab=512, layers=1, theta=500000.0,
               eps=1e-6, slots=2, length=40, positions=64),
    LlamaShape(weights="bf16", cache="bf16"),
    LlamaShape(d_model=512, heads=4, kv_heads=2, head_dim=128, ffn=1024, vocab=3000, layers=2, slots=3, length=96,
               positions=96, weights="bf16", cache="f32"),
    LlamaShape(d_model=512, heads=4, kv_heads=2, head_dim=128, ffn=1024, vocab=3000, layers=2, positions=96,
               blocks=64, block_size=16),
    LlamaShape(layers=32, positions=4096, blocks=4096, block_size=16, weights="bf16", cache="bf16"),
    LlamaShape(weights="f16", cache="f16"),
    LlamaShape(d_model=512, heads=4, kv_heads=2, head_dim=128, ffn=1024, vocab=3000, layers=2, positions=96,
               blocks=64, block_size=16, weights="f16", cache="bf16"),
    LlamaShape(d_model=512, heads=4, kv_heads=4, head_dim=128, ffn=256, vocab=3000, layers=2, slots=2, length=96,
               positions=96, experts=8, top_k=2),
]


def doubled():
    b = program("doubled")
    x = b.input("x", whole_row(4))
    w = b.weight("w", [4, 4])
    y = x
    for k in range(1, 41):
        y = b.add(f"d{k}", y, y)
    b.output("y", b.linear("y", w, 0, y))
    return b.done()


GOLDEN_PROGRAMS = [golden_layer(False), golden_layer(True), golden_head(), two_tiles(), doubled()]


def test_library_exports_the_header():
    L = H.lib()
    header = open(__file__.rsplit("/tests/", 1)[0] + "/include/furykernel_host.h").read()
    import re

    names = re.findall(r"\b(fkh_[a-z_0-9]+)\s*\(", header)
    assert len(names) >= 14
    for n in names:
        assert hasattr(L, n), n
    assert L.fkh_abi_version() == H.ABI_VERSION


@pytest.mark.parametrize("s", SHAPES, ids=range(len(SHAPES)))
@pytest.mark.parametrize("which,build", [("embed", embed_program), ("layer", layer_program),
                                         ("head", head_program)])
def test_llama_programs_render_alike(s, which, build):
    assert H.llama_program_text(s, which) == render_program(build(s))


@pytest.mark.parametrize("i", range(len(GOLDEN_PROGRAMS)))
def test_golden_programs_parse_back(i):
    text = render_program(GOLDEN_PROGRAMS[i])
    assert H.program_roundtrip(text) == text


def test_layer_plan_golden():
    # ProgramTest.hs:559-640, planned by the library.
    assert H.plan_text(render_program(golden_layer(False))) == LAYER_PLAN


@pytest.mark.parametrize("opts", OPTION_SETS, ids=lambda o: f"h{int(o.horizontal)}g{int(o.gated)}"
                         f"s{int(o.store_gelus)}r{o.sequence_rows}")
@pytest.mark.parametrize("i", range(len(GOLDEN_PROGRAMS)))
def test_golden_programs_plan_alike(i, opts):
    p = GOLDEN_PROGRAMS[i]
    got = H.plan_text(render_program(p), opts.horizontal, opts.gated, opts.store_gelus, opts.sequence_rows)
    assert got == PL.render_plan(PL.plan(opts, p))


@pytest.mark.parametrize("s", SHAPES, ids=range(len(SHAPES)))
@pytest.mark.parametrize("rows", [1, 4, 64])
def test_llama_programs_plan_alike(s, rows):
    for build in (embed_program, layer_program, head_program):
        p = build(s)
        assert H.plan_text(render_program(p), sequence_rows=rows) == \
            PL.render_plan(PL.plan(PL.PlanOptions(sequence_rows=rows), p))


def test_refusals_carry_text():
    with pytest.raises(N.Refused, match="expected .program"):
        H.program_roundtrip("nonsense")
    with pytest.raises(N.Refused):
        H.plan_text(render_program(two_tiles()), sequence_rows=0)


def test_text_entry_reports_the_size_it_needs():
    L = H.lib()
    text = render_program(two_tiles()).encode()
    n = ctypes.c_size_t(0)
    buf = ctypes.create_string_buffer(8)
    rc = L.fkh_program_roundtrip(text, buf, 8, ctypes.byref(n), None, 0)
    assert rc == H.FKH_ERR_SPACE and n.value == len(text)


def test_split_for_alike():
    from tests.restated.lowering import split_for

    for n in (1, 512, 4096, 12288, 22016, 32000):
        for k in (64, 1024, 4096, 11008):
            for sms in (132, 148):
                assert H.split_for(n, k, sms) == split_for(n, k, sms)


class Buf:
    """A stand-in device buffer: an address."""

    def __init__(self, ptr):
        self.ptr = ptr

    def __int__(self):
        return self.ptr


def fake_engine(full, batch, rank=0, world=1, peer_exchange=True, fuse_attention=None, sms=148, chunk=32,
                gated=False, store_gelus=False):
    """A Llama with the attributes its launch lists read, at stand-in
    addresses (no device): the same decisions as its constructor."""
    e = object.__new__(Llama)
    s = dataclasses.replace(full, heads=full.heads // world, kv_heads=full.kv_heads // world,
                            ffn=full.ffn // world)
    e.full, e.s, e.m, e.rank, e.world = full, s, batch, rank, world
    e.ctx = SimpleNamespace(sms=sms)
    e.wb, e.cb = (4 if full.weights == "f32" else 2), (4 if full.cache == "f32" else 2)
    e.gate_up_interleaved = batch <= 64
    e.peer_exchange = world > 1 and batch <= 4 and peer_exchange and not s.experts
    e.vocab_local = full.vocab // world
    e.gated, e.store_gelus = gated, store_gelus
    d, qw, kvw, f = s.d_model, s.q_width, s.kv_width, s.ffn
    e.layer_elems = sum(e.layer_sizes())
    at = iter(range(1, 100))
    e.arena = Buf(1 << 44)
    e.kbase, e.vbase = 2 << 44, 3 << 44
    e.ktab = e.vtab = None
    if s.paged:  # the block-address tables
        e.ktab, e.vtab = Buf(5 << 44), Buf((5 << 44) + (1 << 40))
    for name in ("cos", "sin", "tokens", "pos", "slot", "out_ids", "x", "x1", "partial", "qkv", "att", "gu",
                 "act", "logits", "pairs", "pairs_all"):
        setattr(e, name, Buf((4 << 44) + (next(at) << 32)))
    if s.experts:
        e.moe = {name: Buf((8 << 44) + (i << 36)) for i, name in enumerate(
            ("mlp_in", "router_logits", "route_ids", "route_weights", "experts_gu", "experts_act", "experts_out"))}
    e.chunk = chunk
    e.max_splits = (s.positions + chunk - 1) // chunk
    e.part = [Buf((5 << 44) + (i << 32)) for i in range(3)]
    if fuse_attention is None:
        fuse_attention = batch <= 4
    e.fuse_attention = fuse_attention and batch <= 64
    return e


def small(batch, layers=2, d=512, heads=4, ffn=1024, vocab=3000, length=96):
    return LlamaShape(d_model=d, heads=heads, kv_heads=heads, head_dim=128, ffn=ffn, vocab=vocab, layers=layers,
                      slots=batch, length=length, positions=length)


def tp_shape(batch):
    return LlamaShape(d_model=512, heads=8, kv_heads=8, head_dim=128, ffn=1024, vocab=3000, layers=2, slots=batch,
                      length=96, positions=96)


CASES = (
    # the engine's decode tests: batch, fused
    [(small(b), b, 0, 1, True, f) for b, f in ((1, True), (3, True), (2, True), (5, True), (9, True), (20, True),
                                               (3, False), (9, False), (64, None), (65, None), (100, None))]
    # smoke
    + [(LlamaShape(d_model=256, heads=2, kv_heads=2, head_dim=128, ffn=512, vocab=500, layers=2, slots=b,
                   length=64, positions=64), b, 0, 1, True, None) for b in (1, 5)]
    # tensor parallelism: every rank, over peer memory and over NCCL
    + [(tp_shape(b), b, r, w, peer, None) for w in (2, 4, 8) for r in range(w) for b in (1, 3, 16)
       for peer in (True, False)]
    # the bench's configs: the 7B-shaped model at its batches, one and eight ranks
    + [(LlamaShape(layers=32, slots=b, length=2304, positions=2304), b, 0, 1, True, None) for b in (1, 4, 16, 64)]
    + [(LlamaShape(layers=32, slots=1, length=4096, positions=4096), 1, r, 8, True, None) for r in (0, 7)]
    + [(LlamaShape(layers=1, slots=b, length=2304, positions=2304), b, 0, 1, True, f) for b in (1, 16)
       for f in (True, False)]
    # a GQA model over a ring of one slot
    + [(SHAPES[2], 1, 0, 1, True, None),
       (dataclasses.replace(SHAPES[2], slots=4), 4, 0, 1, True, None)]
    + [(SHAPES[2], 1, r, 2, p, None) for r in (0, 1) for p in (True, False)]
    # bf16 weights and bf16 caches: every batch form, fused or not, and tensor parallelism
    + [(dataclasses.replace(small(b), weights="bf16", cache="bf16"), b, 0, 1, True, f)
       for b, f in ((1, None), (3, False), (4, None), (5, None), (9, True), (33, None), (65, None))]
    + [(dataclasses.replace(tp_shape(b), weights="bf16", cache="bf16"), b, r, 4, peer, None) for b in (1, 16)
       for r in (0, 3) for peer in (True, False)]
    + [(dataclasses.replace(small(b), weights=w, cache=c), b, 0, 1, True, None) for b in (1, 8)
       for w, c in (("bf16", "f32"), ("f32", "bf16"))]
    + [(LlamaShape(layers=32, slots=1, length=4096, positions=4096, weights="bf16", cache="bf16"), 1, 0, 1, True,
        None)]
    # paged caches: f32 and bf16, batches of every GEMV form, tensor parallelism
    + [(dataclasses.replace(small(b), blocks=64, block_size=16, cache=c), b, 0, 1, True, None)
       for b in (1, 3, 9, 65) for c in ("f32", "bf16")]
    + [(dataclasses.replace(tp_shape(b), blocks=32, block_size=8), b, r, 2, peer, None) for b in (1, 16)
       for r in (0, 1) for peer in (True, False)]
    # routed experts: a Mixtral-shaped layer, top 2 of 8, and top 1 of 4 over a paged cache
    + [(dataclasses.replace(small(b), experts=8, top_k=2), b, 0, 1, True, None) for b in (1, 3, 9, 32)]
    + [(dataclasses.replace(small(b), experts=4, top_k=1, blocks=32, block_size=16), b, 0, 1, True, None)
       for b in (1, 5)]
    + [(dataclasses.replace(small(b), experts=8, top_k=2, weights="bf16", cache="bf16"), b, 0, 1, True, None)
       for b in (1, 12)]
    # a route with expert scales (a weight of the model's type after the router)
    + [(dataclasses.replace(small(b), experts=8, top_k=2, expert_scale=True, weights=w), b, 0, 1, True, None)
       for b in (1, 9) for w in ("f32", "bf16", "f16")]
    + [(dataclasses.replace(tp_shape(2), ffn=256, experts=8, top_k=2, expert_scale=True), 2, r, 2, False, None)
       for r in (0, 1)]
    # routed experts over ranks: each rank's ffn slice of every expert, the sums by NCCL
    + [(dataclasses.replace(tp_shape(b), ffn=256, experts=8, top_k=2), b, r, w, peer, None) for w in (2, 4)
       for r in (0, w - 1) for b in (1, 5) for peer in (True, False)]
    # f16 weights and f16 caches (and mixed with bf16): every batch form, tensor parallelism, paged, experts
    + [(dataclasses.replace(small(b), weights="f16", cache="f16"), b, 0, 1, True, f)
       for b, f in ((1, None), (3, False), (5, None), (9, True), (65, None))]
    + [(dataclasses.replace(tp_shape(b), weights="f16", cache="f16"), b, r, 2, peer, None) for b in (1, 16)
       for r in (0, 1) for peer in (True, False)]
    + [(dataclasses.replace(small(b), weights=w, cache=c), b, 0, 1, True, None) for b in (1, 8)
       for w, c in (("f16", "bf16"), ("bf16", "f16"), ("f32", "f16"))]
    + [(dataclasses.replace(small(b), blocks=64, block_size=16, weights="f16", cache="f16"), b, 0, 1, True, None)
       for b in (1, 9)]
    + [(dataclasses.replace(small(b), experts=8, top_k=2, weights="f16", cache="f16"), b, 0, 1, True, None)
       for b in (1, 12)]
)


@pytest.mark.parametrize("case", range(len(CASES)))
def test_decode_launches_alike(case):
    full, batch, rank, world, peer, fuse = CASES[case]
    e = fake_engine(full, batch, rank, world, peer, fuse)
    want = RL.decode_launches(e)
    got = e._launches()
    assert [L.kernel for L in got] == [L.kernel for L in want]
    for g, w in zip(got, want):
        assert g.bufs == w.bufs, (g.kernel, g.bufs, w.bufs)
        assert g.params == w.params, (g.kernel, g.params, w.params)
        for k, v in w.params.items():  # floats keep their bits (f32 parameters)
            if isinstance(v, float):
                assert math.isclose(g.params[k], v, rel_tol=0, abs_tol=0) or g.params[k] == v


# The layer's plan options (the reference's optGated and optStoreGelus):
# routed experts with the route, the gate and the routed GEMVs as steps of
# their own.
GATED_CASES = [(dataclasses.replace(small(b), experts=8, top_k=2, weights=w), b, g, sg)
               for b in (1, 5) for w in ("f32", "bf16") for g, sg in ((True, False), (True, True), (False, True))]


@pytest.mark.parametrize("case", range(len(GATED_CASES)))
def test_gated_plans_launch_alike(case):
    full, batch, gated, store_gelus = GATED_CASES[case]
    e = fake_engine(full, batch, gated=gated, store_gelus=store_gelus)
    want = RL.decode_launches(e)
    got = e._launches()
    assert [L.kernel for L in got] == [L.kernel for L in want]
    for g, w in zip(got, want):
        assert g.bufs == w.bufs and g.params == w.params, (g.kernel, g.params, w.params)
    # The same kernels as the default plan's, in the same order: the route,
    # the gate and the routed GEMVs are launched as they were.
    base = fake_engine(full, batch)._launches()
    assert [L.kernel for L in got] == [L.kernel for L in base]


def test_unlowerable_steps_are_refused_alike():
    # A ring of one slot shorter than a batch's rows has staged stores: no kernel.
    full = LlamaShape(d_model=64, heads=4, kv_heads=2, head_dim=8, ffn=48, vocab=40, layers=1, slots=1, length=4,
                      positions=16)
    e = fake_engine(full, 8)
    with pytest.raises(N.Refused):
        RL.decode_launches(e)
    with pytest.raises(N.Refused, match="no kernel runs"):
        e._launches()


def test_uneven_shards_are_refused():
    with pytest.raises(N.Refused, match="does not split over 3 ranks"):
        e = fake_engine(tp_shape(1), 1, 0, 1)
        e.world = 3
        e._launches()


def fake_prefill(eng, rows, chunk=None, positions=None, one_slot=False):
    """A Prefill with the attributes its launch lists read, at stand-in
    addresses: the same decisions as its constructor."""
    from furykernel_b200.prefill import Prefill

    p = object.__new__(Prefill)
    s = eng.s
    p.eng, p.ctx, p.R = eng, eng.ctx, rows
    at = iter(range(1, 100))
    for name in ("w_hi", "w_lo", "rows_buf", "x", "a", "a_hi", "a_lo", "qkv", "att", "tmp", "x1", "gu", "act"):
        setattr(p, name, Buf((6 << 44) + (next(at) << 36)))
    if eng.wb == 4:  # f32 weights: the GEMMs read the weight arena (no TF32 arenas)
        p.w_hi = p.w_lo = None
    p.rs = (rows + 3) // 4 * 4
    p.chunk = chunk or eng.chunk
    p.positions = positions or s.positions
    p.max_splits = (p.positions + p.chunk - 1) // p.chunk
    p.one_slot = one_slot and p.positions <= s.length
    p.part = [Buf((7 << 44) + (i << 36)) for i in range(3)]
    p.moe = {}
    if s.experts:
        p.moe = {n: Buf((9 << 44) + (i << 36)) for i, n in enumerate(
            ("router_logits", "route_ids", "route_weights", "experts_gu", "experts_act", "experts_out"))}
    return p


PREFILL_CASES = (
    # the prefill tests: batch, rows, one slot
    [(small(b), b, 0, 1, True, rows, one, m) for b, rows, one, m in ((1, 128, False, 100), (3, 128, False, 128),
                                                                     (1, 128, True, 64), (3, 128, True, 7))]
    # the bench's prompt prefill (config 5), one and two ranks, and a batch past the interleaved arena
    + [(LlamaShape(layers=4, slots=1, length=4096, positions=4096), 1, r, w, True, 512, True, 512)
       for w in (1, 2) for r in range(w)]
    + [(LlamaShape(layers=2, slots=1, length=4096, positions=4096), 1, 0, 1, True, 512, False, 512)]
    + [(small(65, layers=1), 65, 0, 1, True, 64, False, 33)]
    # tensor parallelism over NCCL and over peer memory
    + [(tp_shape(b), b, r, 4, peer, 32, False, 32) for b in (1, 16) for r in (0, 3) for peer in (True, False)]
    # bf16 weights and caches
    + [(dataclasses.replace(small(b), weights="bf16", cache="bf16"), b, 0, 1, True, 128, one, m)
       for b, one, m in ((1, False, 100), (1, True, 64), (8, False, 128))]
    + [(dataclasses.replace(tp_shape(1), weights="bf16", cache="bf16"), 1, 1, 2, True, 32, False, 32)]
    # paged caches: the split attention over rows, and one prompt through its table
    + [(dataclasses.replace(small(b), blocks=64, block_size=16, cache=c), b, 0, 1, True, 96, one, m)
       for b, one, m, c in ((1, False, 90, "f32"), (1, True, 96, "f32"), (4, True, 50, "bf16"), (8, False, 96, "bf16"))]
    + [(dataclasses.replace(tp_shape(1), blocks=32, block_size=8), 1, 1, 2, True, 32, False, 32)]
    # routed experts: the decode step's kernels over the prompt rows
    + [(dataclasses.replace(small(b), experts=8, top_k=2, weights=w), b, 0, 1, True, rows, one, m)
       for b, rows, one, m, w in ((1, 128, False, 100, "f32"), (2, 128, True, 64, "f32"), (3, 96, False, 96, "bf16"),
                                  (1, 128, False, 70, "f16"))]
    + [(dataclasses.replace(small(4), experts=4, top_k=1, blocks=64, block_size=16), 4, 0, 1, True, 96, True, 50)]
    + [(dataclasses.replace(tp_shape(2), ffn=256, experts=8, top_k=2), 2, r, 2, False, 64, False, 40) for r in (0, 1)]
    + [(dataclasses.replace(small(2), experts=8, top_k=2, expert_scale=True, weights="bf16"), 2, 0, 1, True, 64,
        False, 40)]
    # f16 weights and caches, ring and paged
    + [(dataclasses.replace(small(b), weights="f16", cache="f16"), b, 0, 1, True, 128, one, m)
       for b, one, m in ((1, False, 100), (1, True, 64))]
    + [(dataclasses.replace(small(4), blocks=64, block_size=16, weights="f16", cache="f16"), 4, 0, 1, True, 96,
        True, 50)]
)


@pytest.mark.parametrize("case", range(len(PREFILL_CASES)))
def test_prefill_launches_alike(case):
    full, batch, rank, world, peer, rows, one_slot, m = PREFILL_CASES[case]
    e = fake_engine(full, batch, rank, world, peer)
    e.launches = RL.decode_launches(e)
    # as the bench sizes it: positions up to the prompt's rows
    p = fake_prefill(e, rows, positions=rows if rows == 512 else None, one_slot=one_slot)
    assert p.one_slot == one_slot
    want = RP.prefill_launches(p, m)
    got = p.launches(m)
    assert [L.kernel for L in got] == [L.kernel for L in want]
    for g, w in zip(got, want):
        assert (g.kernel, g.bufs) == (w.kernel, w.bufs)
        assert g.params == w.params, (g.kernel, g.params, w.params)


def test_prefill_rows_are_bounded():
    e = fake_engine(small(1), 1)
    e.launches = RL.decode_launches(e)
    p = fake_prefill(e, 16)
    for m in (0, 17):
        with pytest.raises(N.Refused, match="outside 1..16"):
            p.launches(m)


def test_fused_paged_decode_needs_distinct_table_entries():
    """The fused paged attention stores a row's key while the other rows
    read: the engine takes only tables whose entries are all distinct."""
    full = dataclasses.replace(small(2), blocks=64, block_size=16)
    e = fake_engine(full, 2)
    assert e.fuse_attention
    tables = np.arange(2 * full.table_len, dtype=np.uint32).reshape(2, full.table_len)
    tables[1, 3] = tables[0, 0]  # a block in both rows' tables
    with pytest.raises(N.Refused, match="every block-table entry distinct"):
        e.set_rows(np.array([1, 2], np.uint32), np.array([5, 7], np.uint32), tables)


# Mixtures of the options: element types, paged caches, routed experts with
# scales, gated plans, ranks.
MIXED_CASES = [
    (dataclasses.replace(small(3), experts=8, top_k=2, expert_scale=True, weights="f16", cache="bf16", blocks=64,
                         block_size=16), 3, 0, 1, True, True, False),
    (dataclasses.replace(small(2), experts=8, top_k=2, weights="bf16", cache="f16", blocks=64, block_size=16),
     2, 0, 1, True, True, True),
    (dataclasses.replace(tp_shape(5), ffn=256, experts=8, top_k=2, expert_scale=True, weights="bf16", blocks=48,
                         block_size=8), 5, 1, 2, False, False, True),
    (dataclasses.replace(small(70), experts=4, top_k=1, weights="f16", cache="f16"), 70, 0, 1, True, False, False),
]


@pytest.mark.parametrize("case", range(len(MIXED_CASES)))
def test_mixed_options_launch_alike(case):
    full, batch, rank, world, peer, gated, store_gelus = MIXED_CASES[case]
    e = fake_engine(full, batch, rank, world, peer, gated=gated, store_gelus=store_gelus)
    want, got = RL.decode_launches(e), e._launches()
    assert [L.kernel for L in got] == [L.kernel for L in want]
    for g, w in zip(got, want):
        assert g.bufs == w.bufs and g.params == w.params, (g.kernel, g.params, w.params)
    e.launches = got
    if world == 1:  # and the prefill over the same engine
        p = fake_prefill(e, 64)
        pw, pg = RP.prefill_launches(p, 40), p.launches(40)
        assert [(L.kernel, L.params, L.bufs) for L in pg] == [(L.kernel, L.params, L.bufs) for L in pw]
