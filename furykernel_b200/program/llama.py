"""The Llama-shaped decoder programs of this path, written with the program
builder: one layer (RMSNorm, q/k/v, RoPE, KV store, attention, o, residual,
RMSNorm, SiLU-gated FFN, residual), the embedding, and the head (final
norm, tied LM head, greedy token). All f32: weights, activations and the
Ring KV caches."""

from __future__ import annotations

import math
from dataclasses import dataclass

from .build import program
from .graph import CACHE_F32, AttendTo, AttnSpec, Ring, RopeSpec, StoreAt, whole_row


@dataclass(frozen=True)
class LlamaShape:
    d_model: int = 4096
    heads: int = 32
    kv_heads: int = 32
    head_dim: int = 128
    ffn: int = 11008
    vocab: int = 32000
    layers: int = 32
    theta: float = 10000.0
    eps: float = 1e-5
    slots: int = 1  # sequences the ring holds
    length: int = 4096  # ring length
    positions: int = 4096  # bound of the positions a row may have

    @property
    def q_width(self):
        return self.heads * self.head_dim

    @property
    def kv_width(self):
        return self.kv_heads * self.head_dim


def layer_program(s: LlamaShape, name: str = "layer"):
    """One decoder layer, as a program: the input row x and its position and
    slot in, the layer's output row x out."""
    b = program(name)
    x = b.input("x", whole_row(s.d_model))
    pos = b.row_ints("position", 1, s.positions)
    slot = b.row_ints("slot", 1, s.slots)
    attn_norm = b.weight("attn_norm", [s.d_model], "f32")
    wq = b.weight("q_proj", [s.q_width, s.d_model], "f32")
    wk = b.weight("k_proj", [s.kv_width, s.d_model], "f32")
    wv = b.weight("v_proj", [s.kv_width, s.d_model], "f32")
    wo = b.weight("o_proj", [s.d_model, s.q_width], "f32")
    mlp_norm = b.weight("mlp_norm", [s.d_model], "f32")
    wg = b.weight("gate_proj", [s.ffn, s.d_model], "f32")
    wu = b.weight("up_proj", [s.ffn, s.d_model], "f32")
    wd = b.weight("down_proj", [s.d_model, s.ffn], "f32")
    kc = b.cache("k_cache", Ring(s.slots, s.kv_heads, s.length, s.head_dim), CACHE_F32)
    vc = b.cache("v_cache", Ring(s.slots, s.kv_heads, s.length, s.head_dim), CACHE_F32)
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
    gate = b.linear("gate", wg, 0, m)
    up = b.linear("up", wu, 0, m)
    act = b.silu_mul("mlp_act", gate, up)
    down = b.linear("mlp_out", wd, 0, act)
    x2 = b.add("x2", x1, down)
    b.output("x", x2)
    return b.done()


def embed_program(s: LlamaShape):
    b = program("embed")
    tok = b.row_ints("token", 1, s.vocab)
    table = b.weight("embed", [s.vocab, s.d_model], "f32")
    x = b.gather("x", table, tok, 1.0)
    b.output("x", x)
    return b.done()


def head_program(s: LlamaShape):
    """The final norm, the tied LM head and the greedy token."""
    b = program("head")
    x = b.input("x", whole_row(s.d_model))
    norm = b.weight("final_norm", [s.d_model], "f32")
    embed = b.weight("embed", [s.vocab, s.d_model], "f32")
    n = b.rmsnorm("final_normed", s.eps, norm, 1.0, x)
    logits = b.linear("logits", embed, 0, n)
    token = b.argmax("token", logits)
    b.output("token", token)
    return b.done()
