"""The lowering of planned steps to table launches, on the CPU (addresses
are stand-ins; nothing runs)."""

import pytest

from tests.restated import lowering as E
from furykernel_b200 import target as T
from tests.restated import plan as PL
from furykernel_b200.shape import LlamaShape
from tests.restated.llama import embed_program, head_program, layer_program


def fake_binding(s, m):
    d, qw, kvw, f = s.d_model, s.q_width, s.kv_width, s.ffn
    w, at = {}, 1 << 32
    for name, n in [("q_proj", qw * d), ("k_proj", kvw * d), ("v_proj", kvw * d), ("o_proj", d * qw),
                    ("gate_proj", f * d), ("up_proj", f * d), ("down_proj", d * f), ("attn_norm", d),
                    ("mlp_norm", d), ("embed", s.vocab * d), ("final_norm", d)]:
        w[name] = at
        at += 4 * n
    X, X1, QKV, ATT, GU, LG, ID = (0x1000 * i for i in range(1, 8))
    values = {"x": E.View(X, 0, d, d), "q": E.View(QKV, 0, qw + 2 * kvw, qw),
              "k": E.View(QKV, qw, qw + 2 * kvw, kvw), "v": E.View(QKV, qw + kvw, qw + 2 * kvw, kvw),
              "attended": E.View(ATT, 0, qw, qw), "x1": E.View(X1, 0, d, d), "gate": E.View(GU, 0, 2 * f, f),
              "up": E.View(GU, f, 2 * f, f), "x2": E.View(X, 0, d, d), "logits": E.View(LG, 0, s.vocab, s.vocab),
              "token": E.View(ID, 0, 1, 1)}
    return E.Binding(weights=w, ints={"token": 0x100, "position": 0x200, "slot": 0x300},
                     caches={"k_cache": 0x400, "v_cache": 0x500}, values=values, m=m)


def lowered(s, m):
    b = fake_binding(s, m)
    tables = {"cos": 0x600, "sin": 0x700}
    attn = {"chunk": 128, "max_splits": 32, "partials": [0x800, 0x900, 0xA00]}
    out = []
    for prog in (embed_program(s), layer_program(s), head_program(s)):
        pl = PL.plan(PL.DEFAULT, prog)
        out += [E.lower_step(prog, st, b, tables, attn) for st in pl.steps]
    return out


@pytest.mark.parametrize("m", [1, 16, 32])
def test_llama_steps_lower_to_table_kernels(m):
    s = LlamaShape()
    ls = lowered(s, m)
    assert [L.kernel for L in ls] == ["gather", "gemv_rmsnorm", "kv_store_ring", "attend_split", "attend_combine",
                                      "gemv_add", "gemv_rmsnorm", "gemv_silu_add", "gemv_rmsnorm", "argmax"]
    for L in ls:  # every launch is one the table takes: its dimensions in range
        k = T.SPEC_KERNELS[L.kernel]
        assert set(L.params) == {p.name for p in k.params}, L.kernel
        for p in k.params:
            if p.dim is not None:
                assert p.dim.holds(L.params[p.name]), (L.kernel, p.name, L.params[p.name])
        assert len(L.bufs) == len(k.buffers)
    qkv = ls[1].params
    assert (qkv["n"], qkv["k"]) == (4096 * 3, 4096)
    gu = ls[6].params
    assert (gu["n"], gu["k"]) == (2 * 11008, 4096)
    down = ls[7].params
    assert (down["n"], down["k"], down["up_off"], down["ldx"]) == (4096, 11008, 11008, 2 * 11008)


def test_unsupported_step_is_refused():
    # Staged stores (a ring without room for a step's rows) have no kernel here.
    s = LlamaShape(slots=1, length=4096, positions=4096)
    prog = layer_program(s)
    pl = PL.plan(PL.PlanOptions(sequence_rows=32), prog)
    assert any(w.kind == "Stage" for st in pl.steps for w in st.work)
    b = fake_binding(s, 32)
    with pytest.raises(E.Unlowerable):
        for st in pl.steps:
            E.lower_step(prog, st, b, {"cos": 1, "sin": 2}, {"chunk": 128, "max_splits": 32, "partials": [1, 2, 3]})
