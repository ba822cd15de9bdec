"""Prompt prefill (config 5's prompt): the rows of a prompt through the layers
at once with tcgen05 3xTF32 GEMMs, against the f64 evaluator's bounds; the
pieces it adds to the decode path (interleaved SiLU-gate, attention over a
prompt's rows in one slot) bit for bit with the oracle; and the decode
step that follows, bit for bit with the oracle given the caches prefill
left."""

import math

import numpy as np
import pytest

from oracle import oracle as O
from tests import model_check as MC

pytestmark = pytest.mark.gpu

THREADS = O.threads_default()


@pytest.fixture(scope="module")
def ctx():
    from furykernel_b200 import _native as N

    c = N.Context(0)
    yield c
    c.close()


def same_bits(a, b):
    a = np.ascontiguousarray(a, np.float32).view(np.uint32)
    b = np.ascontiguousarray(b, np.float32).view(np.uint32)
    return a.shape == b.shape and np.array_equal(a, b)


def test_silu_pairs_bits(ctx):
    rows, f = 7, 1000
    x = O.normal(61, rows * 2 * f).reshape(rows, 2 * f)
    dx, dy = ctx.to_device(x), ctx.empty((rows, f))
    ctx.launch("silu_pairs", {"n": rows * f}, [dx, dy])
    want = O.silu_mul(np.ascontiguousarray(x[:, 0::2]), np.ascontiguousarray(x[:, 1::2]))
    assert same_bits(dy.download(), want)
    dx.free()
    dy.free()


@pytest.mark.parametrize("m,heads,kv_heads,length,start", [(70, 4, 2, 96, 0), (300, 4, 4, 512, 0), (1, 2, 1, 64, 0),
                                                           (257, 2, 1, 1024, 700), (129, 3, 1, 2048, 1900)])
def test_prompt_attention_within_bounds(ctx, m, heads, kv_heads, length, start):
    """attend_prompt (query-tiled, for prefill): m rows of one prompt at
    positions start..start+m-1 over the stored keys and values (a prompt
    after `start` earlier positions; one ragged tile of 64 rows; rounds of
    64 positions, the last one partial), within the f64 evaluator's bounds
    and 1e-4 normwise (its orders differ from the split kernel's)."""
    d = 128
    width = (heads + 2 * kv_heads) * d
    qkv = O.normal(91 + m, m * width).reshape(m, width)
    pos = np.arange(start, start + m, dtype=np.uint32)
    slot = np.full(m, 1, np.uint32)
    kc = O.normal(92, 2 * kv_heads * length * d).reshape(2, kv_heads, length, d)
    vc = O.normal(93, 2 * kv_heads * length * d).reshape(2, kv_heads, length, d)
    dq, dkc, dvc, dpos, dslot = (ctx.to_device(a) for a in (qkv, kc, vc, pos, slot))
    dcos, dsin = ctx.rope_tables(10000.0, d, d // 2, length)
    out = ctx.empty((m, heads * d))
    ctx.launch("attend_prompt", {"m": m, "heads": heads, "kv_heads": kv_heads, "d": d, "length": length,
                                 "rotated": d // 2, "ldq": width, "q_off": 0, "ldo": heads * d,
                                 "max_pos": start + m - 1,
                                 "scale": 1.0 / math.sqrt(d)}, [dq, dcos, dsin, dpos, dslot, dkc, dvc, out])
    got = out.download()
    qref = O.r_rope(O.r_input(qkv[:, :heads * d]), d, d // 2, 10000.0, pos)
    ref = O.r_attend(qref, heads, kv_heads, d, length, pos, slot, kc.astype(np.float64), vc.astype(np.float64),
                     1.0 / math.sqrt(d))
    assert O.within(got, ref).all()
    rel = float(np.max(np.abs(got - ref[0])) / np.max(np.abs(ref[0])))
    assert rel <= 1e-4, rel
    for b in (dq, dkc, dvc, dpos, dslot, dcos, dsin, out):
        b.free()


def test_attention_over_prompt_rows(ctx):
    """100 rows of one prompt in one slot, positions 0..99: every row's keys
    and values stored first, then each row over the positions <= its own."""
    m, heads, kv_heads, length, chunk, d = 100, 4, 2, 128, 16, 128
    width = (heads + 2 * kv_heads) * d
    qkv = O.normal(71, m * width).reshape(m, width)
    pos = np.arange(m, dtype=np.uint32)
    slot = np.zeros(m, np.uint32)
    kc = np.zeros((1, kv_heads, length, d), np.float32)
    vc = np.zeros_like(kc)
    cos_t, sin_t = O.rope_tables(10000.0, d, d // 2, length)
    max_splits = (length + chunk - 1) // chunk
    dq, dkc, dvc, dpos, dslot = (ctx.to_device(a) for a in (qkv, kc, vc, pos, slot))
    dcos, dsin = ctx.rope_tables(10000.0, d, d // 2, length)
    pm, pl = ctx.empty(m * heads * max_splits), ctx.empty(m * heads * max_splits)
    pa = ctx.empty(m * heads * max_splits * d)
    out = ctx.empty((m, heads * d))
    ctx.launch("kv_store_ring", {"m": m, "kv_heads": kv_heads, "d": d, "length": length, "rotated": d // 2,
                                 "ldq": width, "k_off": heads * d, "v_off": (heads + kv_heads) * d},
               [dq, dcos, dsin, dpos, dslot, dkc, dvc])
    ctx.launch("attend_split", {"m": m, "heads": heads, "kv_heads": kv_heads, "d": d, "length": length,
                                "rotated": d // 2, "chunk": chunk, "max_splits": max_splits, "ldq": width,
                                "q_off": 0, "scale": 1.0 / math.sqrt(d)},
               [dq, dcos, dsin, dpos, dslot, dkc, dvc, pm, pl, pa])
    ctx.launch("attend_combine", {"m": m, "heads": heads, "d": d, "chunk": chunk, "max_splits": max_splits,
                                  "ldo": heads * d}, [pm, pl, pa, dpos, out])
    kcache, vcache = kc.copy(), vc.copy()
    krot = O.rope(qkv[:, heads * d:(heads + kv_heads) * d], kv_heads, d, d // 2, pos, cos_t, sin_t)
    O.kv_store_ring(krot, kv_heads, d, length, pos, slot, kcache)
    O.kv_store_ring(np.ascontiguousarray(qkv[:, (heads + kv_heads) * d:]), kv_heads, d, length, pos, slot, vcache)
    qrot = O.rope(qkv[:, :heads * d], heads, d, d // 2, pos, cos_t, sin_t)
    want, _ = O.attend(qrot, heads, kv_heads, d, length, pos, slot, kcache, vcache,
                       np.float32(1.0 / math.sqrt(d)), chunk, 4, max_splits, THREADS)
    assert same_bits(out.download(), want)
    for b in (dq, dkc, dvc, dpos, dslot, dcos, dsin, pm, pl, pa, out):
        b.free()


@pytest.mark.parametrize("batch,one_slot", [(1, False), (3, False), (1, True), (3, True)])
def test_prefill_then_decode(ctx, batch, one_slot):
    from furykernel_b200.engine import Llama
    from furykernel_b200.prefill import Prefill
    from furykernel_b200.shape import LlamaShape

    s = LlamaShape(d_model=512, heads=4, kv_heads=4, head_dim=128, ffn=1024, vocab=3000, layers=2, slots=batch,
                   length=96, positions=96)
    eng = Llama(ctx, s, batch, seed=300 + batch, chunk=16)
    pre = Prefill(eng, rows=128, one_slot=one_slot)
    layers, embed, final_norm = MC.host_model(eng)
    lens = [40, 23, 31][:batch]
    prompts = [O.ints(80 + i, n, s.vocab) for i, n in enumerate(lens)]
    slots = np.arange(batch, dtype=np.uint32)
    # Every prompt's rows but its last, all at once (rows of several slots).
    toks = np.concatenate([p[:-1] for p in prompts])
    poss = np.concatenate([np.arange(n - 1, dtype=np.uint32) for n in lens])
    sl = np.concatenate([np.full(n - 1, i, np.uint32) for i, n in enumerate(lens)])
    from furykernel_b200.prefill import prompt_chunks

    for i, n in prompt_chunks(pre, toks, poss, sl):
        pre.run(toks[i:i + n], poss[i:i + n], sl[i:i + n])
    ctx.sync()
    kc_p, vc_p = MC.host_caches(eng)
    # Prefill's stores lie within the f64 evaluator's bounds.
    _, _, stored_ok = MC.referee_decode(eng, layers, embed, final_norm, kc_p, vc_p, toks, poss, sl)
    assert stored_ok
    # The decode step from each prompt's last token: the oracle's bits from
    # the caches prefill left.
    last = np.array([p[-1] for p in prompts], np.uint32)
    lpos = np.array([n - 1 for n in lens], np.uint32)
    eng.set_rows(last, lpos, slots)
    ids = eng.step()
    logits = eng.logits.download()
    want_ids, want_logits, _ = MC.oracle_decode(eng, layers, embed, final_norm, kc_p.copy(), vc_p.copy(), last,
                                                lpos, slots)
    assert same_bits(logits, want_logits)
    assert np.array_equal(ids, want_ids)
    # The whole prompts through the referee: the last rows' logits within
    # its bounds, the greedy ids equal where the bounds decide them.
    kc_f, vc_f = MC.host_caches(eng)
    allt = np.concatenate(prompts)
    allp = np.concatenate([np.arange(n, dtype=np.uint32) for n in lens])
    alls = np.concatenate([np.full(n, i, np.uint32) for i, n in enumerate(lens)])
    ref, (ref_ids, decided), ok = MC.referee_decode(eng, layers, embed, final_norm, kc_f, vc_f, allt, allp, alls)
    assert ok
    rows = np.cumsum(lens) - 1
    assert O.within(logits, (ref[0][rows], ref[1][rows])).all()
    assert np.array_equal(ids[decided[rows]], ref_ids[rows][decided[rows]])
    pre.close()
