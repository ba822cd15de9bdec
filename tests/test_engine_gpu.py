"""A whole decode step through the planner, the lowering, the kernel table and
one CUDA graph, against the oracle: bit for bit with the CPU target's
arithmetic, and within the f64 evaluator's bounds (greedy ids equal where
the bounds decide them)."""

import numpy as np
import pytest

from oracle import oracle as O
from tests import model_check as MC

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    from furykernel_b200 import _native as N

    c = N.Context(0)
    yield c
    c.close()


def small_shape(batch, layers=2, d=512, heads=4, ffn=1024, vocab=3000, length=96):
    from furykernel_b200.shape import LlamaShape

    return LlamaShape(d_model=d, heads=heads, kv_heads=heads, head_dim=128, ffn=ffn, vocab=vocab, layers=layers,
                      slots=batch, length=length, positions=length)


@pytest.mark.parametrize("batch,graph,fused", [(1, True, True), (3, True, True), (2, False, True), (5, True, True),
                                               (9, True, True), (20, False, True), (3, True, False),
                                               (9, False, False)])
def test_small_model_decode_step(ctx, batch, graph, fused):
    from furykernel_b200.engine import Llama

    s = small_shape(batch)
    eng = Llama(ctx, s, batch, seed=100 + batch, chunk=32, prefill_kv=1.0, fuse_attention=fused)
    tokens = O.ints(5 + batch, batch, s.vocab)
    pos = np.array([40, 95, 7][:batch] if batch <= 3 else (np.arange(batch) * 37 + 5) % 96, np.uint32)
    slot = np.arange(batch, dtype=np.uint32)[::-1].copy()
    layers, embed, final_norm = MC.host_model(eng)
    kc0, vc0 = MC.host_caches(eng)
    eng.set_rows(tokens, pos, slot)
    if graph:
        ids = eng.step()
    else:
        eng.run_eager()
        ctx.sync()
        ids = eng.out_ids.download()
    logits = eng.logits.download()
    kc1, vc1 = MC.host_caches(eng)
    kc, vc = kc0.copy(), vc0.copy()
    want_ids, want_logits, want_x = MC.oracle_decode(eng, layers, embed, final_norm, kc, vc, tokens, pos, slot)
    assert np.array_equal(kc1.view(np.uint32), kc.view(np.uint32))
    assert np.array_equal(vc1.view(np.uint32), vc.view(np.uint32))
    assert np.array_equal(eng.x.download().view(np.uint32), want_x.view(np.uint32))
    assert np.array_equal(logits.view(np.uint32), want_logits.view(np.uint32))
    assert np.array_equal(ids, want_ids)
    ref, (ref_ids, decided), stored_ok = MC.referee_decode(eng, layers, embed, final_norm, kc1, vc1, tokens, pos,
                                                           slot)
    assert stored_ok
    assert O.within(logits, ref).all()
    rel = float(np.max(np.abs(logits - ref[0])) / np.max(np.abs(ref[0])))
    assert rel <= 1e-4, rel
    assert np.array_equal(ids[decided], ref_ids[decided])
    # gather; per layer q/k/v, store, attend, combine, o, gate/up, down (the
    # store and attention fused: one launch fewer); head, argmax; advance.
    assert eng.launch_count() == 1 + (6 if fused else 7) * s.layers + 2 + 1


def test_repeated_steps_advance_the_cache(ctx):
    """Greedy decoding: each step's id is the next step's token, the
    position advances; the graph is replayed, not rebuilt."""
    from furykernel_b200.engine import Llama

    s = small_shape(1, layers=1, length=64)
    eng = Llama(ctx, s, 1, seed=7, chunk=16)
    layers, embed, final_norm = MC.host_model(eng)
    kc, vc = MC.host_caches(eng)
    tok = np.array([17], np.uint32)
    for p in range(6):
        eng.set_rows(tok, np.array([p], np.uint32), np.array([0], np.uint32))
        got = eng.step()
        want, _, _ = MC.oracle_decode(eng, layers, embed, final_norm, kc, vc, tok, np.array([p], np.uint32),
                                      np.array([0], np.uint32))
        assert np.array_equal(got, want)
        tok = got
