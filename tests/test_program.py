"""The program layer and the planner against the reference's goldens
(test/Test/FuryKernel/ProgramTest.hs)."""

import math

import pytest

from tests.restated import plan as PL
from tests.restated.build import program
from tests.restated.graph import AttendTo, AttnSpec, Ring, RopeSpec, StoreAt, whole_row


def layer(k_eq_v: bool):
    """ProgramTest.hs:488-557: hidden 32, four query heads of 8 over two KV
    heads, 8 experts of 16 of which a row takes 2."""
    hidden, eps = 32, 1e-6
    b = program("layer_kv" if k_eq_v else "layer")
    x = b.input("x", whole_row(hidden))
    pos = b.row_ints("position", 1, 64)
    slot = b.row_ints("slot", 1, 2)
    pre_attn = b.weight("pre_attn_norm", [hidden])
    wq = b.weight("q_proj", [4 * 8, hidden])
    wk = b.weight("k_proj", [2 * 8, hidden])
    wv = b.weight("v_proj", [2 * 8, hidden])
    q_norm = b.weight("q_norm", [8])
    k_norm = b.weight("k_norm", [8])
    wo = b.weight("o_proj", [hidden, 4 * 8])
    post_attn = b.weight("post_attn_norm", [hidden])
    pre_mlp = b.weight("pre_mlp_norm", [hidden])
    gate_w = b.weight("gate_proj", [48, hidden])
    up_w = b.weight("up_proj", [48, hidden])
    down = b.weight("down_proj", [hidden, 48])
    post_mlp = b.weight("post_mlp_norm", [hidden])
    router_scale = b.weight("router_scale", [hidden])
    router = b.weight("router_proj", [8, hidden])
    expert_scale = b.weight("expert_scale", [8])
    pre_moe = b.weight("pre_moe_norm", [hidden])
    experts_gate_up = b.table("experts_gate_up", 8, [2 * 16, hidden])
    experts_down = b.table("experts_down", 8, [hidden, 16])
    post_moe = b.weight("post_moe_norm", [hidden])
    post_ffn = b.weight("post_ffn_norm", [hidden])
    scalar = b.weight("layer_scalar", [1])
    k_cache = b.cache("k_cache", Ring(2, 2, 12, 8))
    v_cache = b.cache("v_cache", Ring(2, 2, 12, 8))
    a = b.rmsnorm("attn_in", eps, pre_attn, 1, x)
    q = b.linear("q", wq, 8, a)
    k = b.linear("k", wk, 8, a)
    v = k if k_eq_v else b.linear("v", wv, 8, a)
    qn = b.rmsnorm("q_normed", eps, q_norm, 1, q)
    kn = b.rmsnorm("k_normed", eps, k_norm, 1, k)
    vn = b.rmsnorm("v_normed", eps, None, 1, v)
    qr = b.rope("q_rotated", RopeSpec(10000, 4, 1), pos, qn)
    kr = b.rope("k_rotated", RopeSpec(10000, 4, 1), pos, kn)
    b.kv_store("store_k", StoreAt(k_cache.id, pos.id, slot.id), kr)
    b.kv_store("store_v", StoreAt(v_cache.id, pos.id, slot.id), vn)
    o = b.attend("attended", AttnSpec(4, 2, 8, 6, 1.0), qr, AttendTo(k_cache.id, v_cache.id, pos.id, slot.id))
    out = b.linear("attn_out", wo, 0, o)
    out_normed = b.rmsnorm("attn_out_normed", eps, post_attn, 1, out)
    x1 = b.add("x1", x, out_normed)
    bb = b.rmsnorm("mlp_in", eps, pre_mlp, 1, x1)
    gate = b.linear("gate", gate_w, 0, bb)
    up = b.linear("up", up_w, 0, bb)
    r = b.rmsnorm("router_in", eps, router_scale, 1 / math.sqrt(32), x1)
    logits = b.linear("router_logits", router, 0, r)
    g = b.gelu_mul("mlp_act", gate, up)
    ids, ws = b.route("route", 2, expert_scale, logits)
    c = b.rmsnorm("moe_in", eps, pre_moe, 1, x1)
    d = b.linear("mlp_out", down, 0, g)
    gue = b.linear_routed("experts_gate_up_out", experts_gate_up, ids, c)
    ge = b.gated_gelu("experts_act", gue)
    de = b.linear_routed("experts_out", experts_down, ids, ge)
    h1 = b.rmsnorm("mlp_out_normed", eps, post_mlp, 1, d)
    s = b.combine_ranks("experts_sum", ws, de)
    h2 = b.rmsnorm("moe_out_normed", eps, post_moe, 1, s)
    hs = b.add("ffn_sum", h1, h2)
    f = b.rmsnorm("ffn_out", eps, post_ffn, 1, hs)
    x2 = b.add("x2_unscaled", x1, f)
    y = b.scale_by("x2", scalar, x2)
    b.output("x", y)
    return b.done()


# ProgramTest.hs:559-640.
LAYER_PLAN = """plan layer
  step s0_gemv
    recompute attn_in
    anchor q
    anchor k
    anchor v
    reads x f32
    stores q f32
    stores k f32
    stores v f32
  step s1_store
    recompute k_normed
    recompute v_normed
    recompute k_rotated
    effect store_k
    effect store_v
    reads k f32
    reads v f32
  step s2_attend
    recompute q_normed
    recompute q_rotated
    anchor attended
    reads q f32
    stores attended partials
  step s3_combine
    combine attended
    reads attended partials
    stores attended f32
  step s4_gemv
    anchor attn_out
    reads attended f32
    stores attn_out f32
  step s5_gemv
    recompute attn_out_normed
    recompute x1
    recompute mlp_in
    anchor gate
    anchor up
    recompute router_in
    anchor router_logits
    reads x f32
    reads attn_out f32
    stores x1 f32
    stores gate f32
    stores up f32
    stores router_logits f32
  step s6_gemv
    recompute mlp_act
    recompute route_ids
    recompute moe_in
    anchor mlp_out
    anchor experts_gate_up_out
    reads x1 f32
    reads gate f32
    reads up f32
    reads router_logits f32
    stores route_ids u32
    stores route_weights f32
    stores mlp_out f32
    stores experts_gate_up_out f32
  step s7_gemv
    recompute experts_act
    anchor experts_out
    reads route_ids u32
    reads experts_gate_up_out f32
    stores experts_out f32
  step s8_x2
    recompute mlp_out_normed
    recompute experts_sum
    recompute moe_out_normed
    recompute ffn_sum
    recompute ffn_out
    recompute x2_unscaled
    recompute x2
    reads x1 f32
    reads route_weights f32
    reads mlp_out f32
    reads experts_out f32
    stores x2 f32
"""


def test_layer_plan_golden():
    assert PL.render_plan(PL.plan(PL.DEFAULT, layer(False))) == LAYER_PLAN


def head_program():
    """ProgramTest.hs:642-652: final norm, tied unembedding, softcap, greedy token."""
    b = program("head")
    x = b.input("x", whole_row(32))
    norm = b.weight("final_norm", [32])
    embed = b.weight("embed", [64, 32])
    n = b.rmsnorm("final_normed", 1e-6, norm, 1, x)
    logits = b.linear("logits", embed, 0, n)
    capped = b.softcap("capped", 30, logits)
    token = b.argmax("token", capped)
    b.output("token", token)
    return b.done()


def two_tiles():
    b = program("two_tiles")
    x = b.input("x", whole_row(32))
    wa = b.weight("wa", [16, 32])
    wb = b.weight("wb", [16, 32])
    a = b.linear("a", wa, 0, x)
    c = b.linear("b", wb, 0, x)
    s = b.add("c", a, c)
    b.output("c", s)
    return b.done()


OPTION_SETS = [PL.PlanOptions(h, g, s, r) for h in (True, False) for g in (False, True) for s in (False, True)
               for r in (1, 64)]


@pytest.mark.parametrize("prog", [layer(False), layer(True), head_program(), two_tiles()])
@pytest.mark.parametrize("opts", OPTION_SETS)
def test_plans_are_well_formed(prog, opts):
    """PlanCheck.hs's independent checks, restated: every node runs in some
    step; a step reads only what earlier steps stored or inputs; the
    program's outputs are stored; step names are step names."""
    pl = PL.plan(opts, prog)
    done = set()
    stored = {}
    for s in pl.steps:
        assert PL.is_step_name(s.name), s.name
        for st in s.reads:
            prod = prog.producer_of(st.value)
            assert prod.op.kind == "Input" or (st.value, st.form) in stored, (s.name, st)
        for w in s.work:
            done.add(w.node)
        for st in s.stores:
            stored[(st.value, st.form)] = s.index
    assert {n.id for n in prog.nodes if n.op.kind != "Input"} <= done
    for o in prog.outputs:
        assert any(v == o.value for v, _ in stored)


def test_head_plan():
    # ProgramTest.hs:88-101: softcap on the tiles, argmax a light step after them.
    text = PL.render_plan(PL.plan(PL.DEFAULT, head_program()))
    assert text.splitlines() == [
        "plan head", "  step s0_gemv", "    recompute final_normed", "    anchor logits", "    epilogue capped",
        "    reads x f32", "    stores capped f32", "  step s1_token", "    recompute token", "    reads capped f32",
        "    stores token u32"]


def test_two_tiles_golden():
    # ProgramTest.hs:131-146: elementwise work on two anchors' tiles waits for them.
    assert PL.render_plan(PL.plan(PL.DEFAULT, two_tiles())).splitlines() == [
        "plan two_tiles", "  step s0_gemv", "    anchor a", "    anchor b", "    reads x f32", "    stores a f32",
        "    stores b f32", "  step s1_c", "    recompute c", "    reads a f32", "    reads b f32", "    stores c f32"]
    pl = PL.plan(PL.PlanOptions(horizontal=False), two_tiles())
    # Apart, b joins no step, and c runs as an epilogue on b's tile.
    assert [s.name for s in pl.steps] == ["s0_gemv", "s1_gemv"]


def test_forty_doublings_planned_once():
    # ProgramTest.hs:109-115: a value reached by many paths is planned over each node once.
    b = program("doubled")
    x = b.input("x", whole_row(4))
    w = b.weight("w", [4, 4])
    y = x
    for k in range(1, 41):
        y = b.add(f"d{k}", y, y)
    b.output("y", b.linear("y", w, 0, y))
    pl = PL.plan(PL.DEFAULT, b.done())
    assert [(s.name, len(s.work)) for s in pl.steps] == [("s0_gemv", 41)]


def test_render_program_golden():
    # ProgramTest.hs:116-125.
    from tests.restated.graph import render_program

    b = program("small")
    x = b.input("x", whole_row(4))
    w = b.weight("w", [4, 4])
    y = b.linear("y", w, 0, x)
    n = b.rmsnorm("n", 1e-6, None, 1, y)
    b.output("n", n)
    assert render_program(b.done()).splitlines() == [
        "program small", "  source x : input [4/4] f32", "  source w : weight [4, 4] bf16 out_in",
        "  x : [4/4] f32 = x input(x)", "  y : [4/4] f32 = y linear(w, x) segment 4",
        "  n : [4/4] f32 = n rmsnorm(y, eps f64:0x3eb0c6f7a0b5ed8d, factor f64:0x3ff0000000000000)",
        "  output n = n"]


def test_step_names():
    assert PL.is_step_name("s0_x") and PL.is_step_name("s12_combine")
    assert not PL.is_step_name("s_x") and not PL.is_step_name("s0_") and not PL.is_step_name("x0_y")


# ---------------------------------------------------------------------------
# More of ProgramTest.hs's goldens (ProgramTest.hs:46-86, :113-127), for the
# Python planner and the C++ host library's alike.


def predicting():
    """ProgramTest.hs:769-782: a route the program outputs beside the experts'."""
    b = program("predicting")
    x = b.input("x", whole_row(32))
    router = b.weight("router_proj", [8, 32])
    ahead = b.weight("ahead_proj", [8, 32])
    experts = b.table("experts", 8, [16, 32])
    logits = b.linear("router_logits", router, 0, x)
    ahead_logits = b.linear("ahead_logits", ahead, 0, x)
    ids, ws = b.route("route", 2, None, logits)
    ahead_ids, _ = b.route("ahead", 2, None, ahead_logits)
    y = b.linear_routed("experts_out", experts, ids, x)
    s = b.combine_ranks("experts_sum", ws, y)
    b.output("y", s)
    b.output("ahead", ahead_ids)
    return b.done()


def embed_program():
    """ProgramTest.hs:785-790: tokens to the residual stream, scaled."""
    b = program("embed")
    tokens = b.row_ints("tokens", 1, 64)
    embed = b.weight("embed", [64, 32])
    x = b.gather("x", embed, tokens, 5.65625)
    b.output("x", x)
    return b.done()


def names_both(prog, opts):
    from furykernel_b200 import _host as H
    from tests.restated.graph import render_program

    py = [s.name for s in PL.plan(opts, prog).steps]
    text = H.plan_text(render_program(prog), opts.horizontal, opts.gated, opts.store_gelus, opts.sequence_rows)
    cc = [ln.split()[1] for ln in text.splitlines() if ln.startswith("  step ")]
    assert py == cc
    return py


def test_keys_as_values_plan_the_same_without_the_value_projection():
    assert names_both(layer(True), PL.DEFAULT) == ["s0_gemv", "s1_store", "s2_attend", "s3_combine", "s4_gemv",
                                                   "s5_gemv", "s6_gemv", "s7_gemv", "s8_x2"]


def test_stored_gelus_and_gated_routes():
    assert names_both(layer(False), PL.PlanOptions(store_gelus=True)) == [
        "s0_gemv", "s1_store", "s2_attend", "s3_combine", "s4_gemv", "s5_gemv", "s6_mlp_act", "s7_gemv",
        "s8_experts_act", "s9_gemv", "s10_x2"]
    assert names_both(layer(False), PL.PlanOptions(gated=True, store_gelus=True)) == [
        "s0_gemv", "s1_store", "s2_attend", "s3_combine", "s4_gemv", "s5_gemv", "s6_route_ids", "s7_gemv",
        "s8_gemv", "s9_experts_act", "s10_gemv", "s11_x2"]
    assert names_both(layer(False), PL.PlanOptions(gated=True)) == [
        "s0_gemv", "s1_store", "s2_attend", "s3_combine", "s4_gemv", "s5_gemv", "s6_route_ids", "s7_gemv",
        "s8_gemv", "s9_gemv", "s10_x2"]


def test_gated_a_route_the_program_outputs_is_stored_beside_the_experts_route():
    from furykernel_b200 import _host as H
    from tests.restated.graph import render_program

    want = [
        "plan predicting",
        "  step s0_gemv",
        "    anchor router_logits",
        "    anchor ahead_logits",
        "    reads x f32",
        "    stores router_logits f32",
        "    stores ahead_logits f32",
        "  step s1_route_ids",
        "    recompute route_ids",
        "    recompute ahead_ids",
        "    reads router_logits f32",
        "    reads ahead_logits f32",
        "    stores route_ids u32",
        "    stores route_weights f32",
        "    stores ahead_ids u32",
        "  step s2_gemv",
        "    anchor experts_out",
        "    reads x f32",
        "    reads route_ids u32",
        "    stores experts_out f32",
        "  step s3_experts_sum",
        "    recompute experts_sum",
        "    reads route_weights f32",
        "    reads experts_out f32",
        "    stores experts_sum f32",
    ]
    opts = PL.PlanOptions(gated=True)
    assert PL.render_plan(PL.plan(opts, predicting())).splitlines() == want
    assert H.plan_text(render_program(predicting()), True, True, False, 1).splitlines() == want


def test_the_embedding_one_light_step():
    from furykernel_b200 import _host as H
    from tests.restated.graph import render_program

    want = ["plan embed", "  step s0_x", "    recompute x", "    stores x f32"]
    assert PL.render_plan(PL.plan(PL.DEFAULT, embed_program())).splitlines() == want
    assert H.plan_text(render_program(embed_program())).splitlines() == want
    # A step's kernel name splits back at the first _x_ whose right side is
    # a step's name (ProgramTest.hs:103-109); "" asks for that rule.
    left, _ = H.split_join("embed_x_s0_x_x_m1", "m")
    assert H.split_join(left, "") == ("embed", "s0_x")
    assert H.split_join("embed_x_s0_x", "") == ("embed", "s0_x")
    assert H.split_join("embed_x_x_s1_store", "") == ("embed_x", "s1_store")
    assert [PL.is_step_name(t) for t in ["s0_x", "s12_attend", "s_x", "s0", "s0_", "x0_s"]] == \
        [True, True, False, False, False, False]
