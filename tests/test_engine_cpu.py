"""Host-side logic of the engine and the prefill that needs no GPU: the
rewrite of a decode step's KV store and attention into one launch, the
prompt rows a prefill takes and the runs it takes them in."""

from types import SimpleNamespace

import numpy as np

from furykernel_b200.engine import Launch, Llama
from furykernel_b200.prefill import prompt_chunks, prompt_rows
from tests.restated import lowering as RL


def kv_launch(qkv=100, pos=200, slot=300, kc=400, vc=500, ldq=1536, rotated=64, length=96):
    return Launch("kv_store_ring", {"m": 2, "kv_heads": 4, "d": 128, "length": length, "rotated": rotated,
                                    "ldq": ldq, "k_off": 512, "v_off": 1024},
                  [qkv, 11, 12, pos, slot, kc, vc])


def attend_launch(qkv=100, pos=200, slot=300, kc=400, vc=500, ldq=1536, rotated=64, length=96):
    return Launch("attend_split", {"m": 2, "heads": 4, "kv_heads": 4, "d": 128, "length": length,
                                   "rotated": rotated, "chunk": 16, "max_splits": 6, "ldq": ldq, "q_off": 0,
                                   "scale": 0.08838834764831845},
                  [qkv, 11, 12, pos, slot, kc, vc, 21, 22, 23])


def test_fuse_attention_merges_a_store_and_its_attention():
    combine = Launch("attend_combine", {"m": 2}, [21, 22, 23, 200, 600])
    out = RL.fuse_attention(SimpleNamespace(), [Launch("gemv", {}, []), kv_launch(), attend_launch(), combine])
    assert [L.kernel for L in out] == ["gemv", "attend_decode", "attend_combine"]
    fused = out[1]
    assert fused.bufs == attend_launch().bufs
    assert fused.params["k_off"] == 512 and fused.params["v_off"] == 1024
    assert {k: v for k, v in fused.params.items() if k not in ("k_off", "v_off")} == attend_launch().params


def test_fuse_attention_leaves_mismatched_launches():
    for kw in ({"qkv": 101}, {"slot": 301}, {"kc": 401}, {"ldq": 1540}, {"rotated": 32}, {"length": 64}):
        launches = [kv_launch(**kw), attend_launch()]
        out = RL.fuse_attention(SimpleNamespace(), launches)
        assert [L.kernel for L in out] == ["kv_store_ring", "attend_split"], kw


def test_prompt_rows_drop_each_prompt_s_last_row():
    toks, poss, sl = prompt_rows([[5, 6, 7], [8, 9]], [3, 1])
    assert toks.tolist() == [5, 6, 8]
    assert poss.tolist() == [0, 1, 0]
    assert sl.tolist() == [3, 3, 1]


def test_prompt_chunks_respect_the_row_budget_and_slots():
    toks, poss, sl = prompt_rows([np.arange(8), np.arange(4), np.arange(7)], [0, 1, 2])
    mixed = SimpleNamespace(R=5, one_slot=False)
    assert prompt_chunks(mixed, toks, poss, sl) == [(0, 5), (5, 5), (10, 5), (15, 1)]
    one = SimpleNamespace(R=5, one_slot=True)
    runs = prompt_chunks(one, toks, poss, sl)
    assert runs == [(0, 5), (5, 2), (7, 3), (10, 5), (15, 1)]
    for i, m in runs:
        assert len(set(sl[i:i + m].tolist())) == 1
    assert sum(m for _, m in runs) == len(toks)


def test_row_inputs_past_the_engine_s_tables_are_refused():
    from furykernel_b200 import _native as N

    eng = SimpleNamespace(s=SimpleNamespace(positions=64, slots=2, paged=False, blocks=0),
                          full=SimpleNamespace(vocab=100))
    Llama.check_rows(eng, [1, 99], [0, 63], [0, 1])
    for tokens, pos, slots, what in (([100], [0], [0], "token 100"), ([1], [64], [0], "position 64"),
                                     ([1], [0], [2], "slot 2")):
        try:
            Llama.check_rows(eng, tokens, pos, slots)
        except N.Refused as e:
            assert what in str(e)
        else:
            raise AssertionError(what)
    # A paged cache: every block-table entry within the pool.
    paged = SimpleNamespace(s=SimpleNamespace(positions=64, slots=1, paged=True, blocks=8),
                            full=SimpleNamespace(vocab=100))
    Llama.check_rows(paged, [1, 2], [0, 63], [[0, 1, 2, 3], [7, 6, 5, 4]])
    try:
        Llama.check_rows(paged, [1], [0], [[0, 8, 1, 2]])
    except N.Refused as e:
        assert "block 8" in str(e)
    else:
        raise AssertionError("block 8")
