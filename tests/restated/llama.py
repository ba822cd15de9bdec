"""Test infrastructure: the Python restatement that the C++ host library
(libfurykernel_host.so) is checked against. The Llama-shaped decoder
programs of this path, written with the program builder: one layer (RMSNorm, q/k/v, RoPE, KV store, attention, o, residual,
RMSNorm, SiLU-gated FFN, residual), the embedding, and the head (final
norm, tied LM head, greedy token). Activations are f32; the weights and the
KV caches are f32 (the BASELINE configurations), bf16 (the reference's own
element types) or f16."""

from __future__ import annotations

import math

from furykernel_b200.shape import LlamaShape

from .build import program
from .graph import AttendTo, AttnSpec, Paged, Ring, RopeSpec, StoreAt, whole_row


def layer_program(s: LlamaShape, name: str = "layer"):
    """One decoder layer, as a program: the input row x and its position and
    slot in, the layer's output row x out."""
    b = program(name)
    x = b.input("x", whole_row(s.d_model))
    pos = b.row_ints("position", 1, s.positions)
    # A row's sequence: its slot of the ring, or its block table of the pool.
    slot = b.row_ints("block_table", s.table_len, s.blocks) if s.paged else b.row_ints("slot", 1, s.slots)
    attn_norm = b.weight("attn_norm", [s.d_model], s.weights)
    wq = b.weight("q_proj", [s.q_width, s.d_model], s.weights)
    wk = b.weight("k_proj", [s.kv_width, s.d_model], s.weights)
    wv = b.weight("v_proj", [s.kv_width, s.d_model], s.weights)
    wo = b.weight("o_proj", [s.d_model, s.q_width], s.weights)
    mlp_norm = b.weight("mlp_norm", [s.d_model], s.weights)
    # The dense FFN's weights, or the router and the experts' tables.
    if s.experts:
        router = b.weight("router", [s.experts, s.d_model], s.weights)
        scale = b.weight("expert_scale", [s.experts], s.weights) if s.expert_scale else None
        egu = b.table("experts_gate_up", s.experts, [2 * s.ffn, s.d_model], s.weights)
        edn = b.table("experts_down", s.experts, [s.d_model, s.ffn], s.weights)
    else:
        wg = b.weight("gate_proj", [s.ffn, s.d_model], s.weights)
        wu = b.weight("up_proj", [s.ffn, s.d_model], s.weights)
        wd = b.weight("down_proj", [s.d_model, s.ffn], s.weights)
    layout = Paged(s.blocks, s.block_size, s.kv_heads, s.head_dim) if s.paged else \
        Ring(s.slots, s.kv_heads, s.length, s.head_dim)
    kc = b.cache("k_cache", layout, s.cache)
    vc = b.cache("v_cache", layout, s.cache)
    a = b.rmsnorm("attn_in", s.eps, attn_norm, 1.0, x)
    q = b.linear("q", wq, s.head_dim, a)
    k = b.linear("k", wk, s.head_dim, a)
    v = b.linear("v", wv, s.head_dim, a)
    rope = RopeSpec(s.theta, s.head_dim // 2, 1)
    qr = b.rope("q_rotated", rope, pos, q)
    kr = b.rope("k_rotated", rope, pos, k)
    b.kv_store("store_k", StoreAt(kc.id, pos.id, slot.id), kr)
    b.kv_store("store_v", StoreAt(vc.id, pos.id, slot.id), v)
    o = b.attend("attended", AttnSpec(s.heads, s.kv_heads, s.head_dim, None, 1.0 / math.sqrt(s.head_dim)), qr,
                 AttendTo(kc.id, vc.id, pos.id, slot.id))
    out = b.linear("attn_out", wo, 0, o)
    x1 = b.add("x1", x, out)
    m = b.rmsnorm("mlp_in", s.eps, mlp_norm, 1.0, x1)
    if s.experts:  # each row's top_k experts, GELU-gated, weighted by the route
        logits = b.linear("router_logits", router, 0, m)
        ids, ws = b.route("route", s.top_k, scale, logits)
        gu = b.linear_routed("experts_gu", egu, ids, m)
        act = b.gated_gelu("experts_act", gu)
        eo = b.linear_routed("experts_out", edn, ids, act)
        ffn_out = b.combine_ranks("experts_sum", ws, eo)
    else:
        gate = b.linear("gate", wg, 0, m)
        up = b.linear("up", wu, 0, m)
        act = b.silu_mul("mlp_act", gate, up)
        ffn_out = b.linear("mlp_out", wd, 0, act)
    x2 = b.add("x2", x1, ffn_out)
    b.output("x", x2)
    return b.done()


def embed_program(s: LlamaShape):
    b = program("embed")
    tok = b.row_ints("token", 1, s.vocab)
    table = b.weight("embed", [s.vocab, s.d_model], s.weights)
    x = b.gather("x", table, tok, 1.0)
    b.output("x", x)
    return b.done()


def head_program(s: LlamaShape):
    """The final norm, the tied LM head and the greedy token."""
    b = program("head")
    x = b.input("x", whole_row(s.d_model))
    norm = b.weight("final_norm", [s.d_model], s.weights)
    embed = b.weight("embed", [s.vocab, s.d_model], s.weights)
    n = b.rmsnorm("final_normed", s.eps, norm, 1.0, x)
    logits = b.linear("logits", embed, 0, n)
    token = b.argmax("token", logits)
    b.output("token", token)
    return b.done()
