"""Parity of the routed-expert kernels on a B200, through the C ABI: the
route, the expert-grouped routed GEMV, the GELU-tanh gate and the
rank-weighted combine, each bit for bit with the oracle's restatement
(oracle/fko_cpu.c), and a decode step of a model whose FFN is routed
experts, bit for bit with the oracle's decode."""


import numpy as np
import pytest

from furykernel_b200.target import WEIGHT_SUFFIX
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


@pytest.mark.parametrize("m,n,k", [(1, 8, 2), (3, 64, 4), (16, 1000, 8), (5, 4, 4)])
def test_route_topk(ctx, m, n, k):
    x = O.normal(201, m * n).reshape(m, n)
    x[0, : min(3, n)] = 1.5  # ties: the lower index first
    xd, ids, ws = ctx.to_device(x), ctx.zeros((m, k), np.uint32), ctx.zeros((m, k))
    ctx.launch("route_topk", {"m": m, "n": n, "k": k, "ldx": n}, [xd, ids, ws])
    want_ids, want_ws = O.route_topk(x, k)
    assert np.array_equal(ids.download(), want_ids)
    assert same_bits(ws.download(), want_ws)
    scale = O.uniform(202, n, 0.5, 1.5)
    sd = ctx.to_device(scale)
    ctx.launch("route_topk_scaled", {"m": m, "n": n, "k": k, "ldx": n}, [xd, sd, ids, ws])
    want_ids, want_ws = O.route_topk(x, k, scale)
    assert np.array_equal(ids.download(), want_ids) and same_bits(ws.download(), want_ws)
    for t in ("bf16", "f16"):  # scales of the weights' 16-bit type, widened where read
        bits = MC.narrow(t, scale)
        bd = ctx.to_device(bits)
        ctx.launch("route_topk_scaled" + WEIGHT_SUFFIX[t], {"m": m, "n": n, "k": k, "ldx": n}, [xd, bd, ids, ws])
        want_ids, want_ws = O.route_topk(x, k, MC.widen(t, bits))
        assert np.array_equal(ids.download(), want_ids) and same_bits(ws.download(), want_ws)
        bd.free()
    for b in (xd, ids, ws, sd):
        b.free()


@pytest.mark.parametrize("entries,n,kk,m,k,split", [(8, 2048, 512, 3, 2, 1), (8, 512, 1024, 3, 2, 2),
                                                    (64, 1408, 2048, 16, 4, 1), (4, 256, 256, 8, 8, 4)])
def test_gemv_routed_shared_and_per_rank(ctx, entries, n, kk, m, k, split):
    table = O.normal(211, entries * n * kk, 0.0, 0.02).reshape(entries, n, kk)
    ids = O.ints(212, m * k, entries).reshape(m, k).astype(np.uint32)
    td, idd = ctx.to_device(table), ctx.to_device(ids)
    for per_rank in (0, 1):
        xw = k * kk if per_rank else kk
        x = O.normal(213 + per_rank, m * xw).reshape(m, xw)
        xd, yd = ctx.to_device(x), ctx.zeros((m, k * n))
        ctx.launch("gemv_routed", {"entries": entries, "n": n, "kk": kk, "m": m, "k": k, "split": split, "ldx": xw,
                                   "ldy": k * n, "per_rank": per_rank}, [td, idd, xd, yd])
        assert same_bits(yd.download(), O.gemv_routed(table, ids, x, split, THREADS))
        # The 16-bit table forms: the f32 arithmetic over the widened entries.
        for t in ("bf16", "f16"):
            bits = MC.narrow(t, table).reshape(table.shape)
            bd = ctx.to_device(bits)
            ctx.launch("gemv_routed" + WEIGHT_SUFFIX[t], {"entries": entries, "n": n, "kk": kk, "m": m, "k": k,
                                                         "split": split, "ldx": xw, "ldy": k * n,
                                                         "per_rank": per_rank}, [bd, idd, xd, yd])
            widened = MC.widen(t, bits).reshape(table.shape)
            assert same_bits(yd.download(), O.gemv_routed(widened, ids, x, split, THREADS))
            bd.free()
        for b in (xd, yd):
            b.free()
    td.free()
    idd.free()


def test_gated_gelu_and_combine(ctx):
    m, k, f, d = 5, 4, 1024, 512
    gu = O.normal(221, m * k * 2 * f, 0.0, 2.0).reshape(m, k * 2 * f)
    gd, ad = ctx.to_device(gu), ctx.zeros((m, k * f))
    ctx.launch("gated_gelu", {"segments": m * k, "f": f}, [gd, ad])
    assert same_bits(ad.download(), O.gated_gelu(gu, f))
    r = O.normal(222, m * d).reshape(m, d)
    ws = O.uniform(223, m * k, 0.0, 1.0).reshape(m, k)
    segs = O.normal(224, m * k * d).reshape(m, k * d)
    rd, wd, sd, yd = ctx.to_device(r), ctx.to_device(ws), ctx.to_device(segs), ctx.zeros((m, d))
    ctx.launch("combine_ranks_add", {"m": m, "k": k, "d": d}, [rd, wd, sd, yd])
    assert same_bits(yd.download(), O.combine_ranks_add(r, ws, segs))
    for b in (gd, ad, rd, wd, sd, yd):
        b.free()


@pytest.mark.parametrize("batch,experts,top_k,weights,gated,store_gelus", [
    (1, 8, 2, "f32", False, False), (3, 8, 2, "f32", False, False), (9, 16, 4, "f32", False, False),
    (2, 8, 2, "bf16", False, False), (12, 8, 2, "bf16", False, False), (5, 8, 2, "f16", False, False),
    (3, 8, 2, "f32", True, False), (3, 8, 2, "f32", True, True), (4, 8, 2, "bf16", False, True),
    (3, 8, 2, "f32", "scale", False), (2, 8, 2, "bf16", "scale", False)])
def test_moe_model_decode_step(ctx, batch, experts, top_k, weights, gated, store_gelus):
    """A decode step of a model whose FFN is routed experts, captured as a
    graph, against the oracle's decode: the same ids, logits and residual
    rows, bit for bit -- with the default plan, and with the route and the
    gate in steps of their own (optGated, optStoreGelus)."""
    from furykernel_b200.engine import Llama
    from furykernel_b200.shape import LlamaShape

    scaled = gated == "scale"  # the route's expert scales, the default plan
    gated = gated is True
    s = LlamaShape(d_model=512, heads=4, kv_heads=4, head_dim=128, ffn=256, vocab=3000, layers=2, slots=batch,
                   length=96, positions=96, experts=experts, top_k=top_k, weights=weights, expert_scale=scaled)
    eng = Llama(ctx, s, batch, seed=500 + batch, chunk=32, prefill_kv=1.0, gated=gated, store_gelus=store_gelus)
    tokens = O.ints(29 + batch, batch, s.vocab)
    pos = ((np.arange(batch) * 37 + 5) % 96).astype(np.uint32)
    slot = np.arange(batch, dtype=np.uint32)
    layers, embed, final_norm = MC.host_model(eng)
    kc, vc = MC.host_caches(eng)
    eng.set_rows(tokens, pos, slot)
    ids = eng.step()
    want_ids, want_logits, want_x = MC.oracle_decode(eng, layers, embed, final_norm, kc, vc, tokens, pos, slot)
    assert np.array_equal(ids, want_ids)
    assert same_bits(eng.logits.download(), want_logits)
    assert same_bits(eng.x.download(), want_x)


@pytest.mark.parametrize("weights,one_slot", [("f32", False), ("f32", True), ("bf16", False)])
def test_moe_prefill(ctx, weights, one_slot):
    """Prefill of a model whose FFN is routed experts: the last layer's
    experts over the prompt rows are the decode step's kernels, so from the
    rows prefill left (the attention residual and its norm) the oracle
    gives their logits, route, outputs and the layer's output bit for bit;
    the decode step from the caches prefill left is the oracle's too."""
    from furykernel_b200.engine import Llama
    from furykernel_b200.prefill import Prefill, prompt_chunks
    from furykernel_b200.shape import LlamaShape

    batch = 2
    s = LlamaShape(d_model=512, heads=4, kv_heads=4, head_dim=128, ffn=256, vocab=3000, layers=2, slots=batch,
                   length=96, positions=96, experts=8, top_k=2, weights=weights)
    eng = Llama(ctx, s, batch, seed=520, chunk=16)
    pre = Prefill(eng, rows=128, one_slot=one_slot)
    layers, embed, final_norm = MC.host_model(eng)
    lens = [41, 30]
    prompts = [O.ints(230 + i, n, s.vocab) for i, n in enumerate(lens)]
    toks = np.concatenate([p[:-1] for p in prompts])
    poss = np.concatenate([np.arange(n - 1, dtype=np.uint32) for n in lens])
    sl = np.concatenate([np.full(n - 1, i, np.uint32) for i, n in enumerate(lens)])
    runs = prompt_chunks(pre, toks, poss, sl)
    for i, n in runs:
        pre.run(toks[i:i + n], poss[i:i + n], sl[i:i + n])
    ctx.sync()
    # The last run's last layer, recomputed from its attention residual.
    m = runs[-1][1]
    w = layers[-1]
    d = s.d_model
    x1 = pre.x1.download()[:m]
    a = O.rmsnorm_rows(x1, w["mlp_norm"], np.float32(s.eps), 1.0, THREADS)
    assert same_bits(pre.a.download()[:m], a)
    logits = O.gemv(w["router"], a, 1, THREADS)
    assert same_bits(pre.moe["router_logits"].download()[:m], logits)
    ids, ws = O.route_topk(logits, s.top_k)
    assert np.array_equal(pre.moe["route_ids"].download()[:m], ids)
    gu = O.gemv_routed(w["egu"], ids, a, 1, THREADS)
    eo = O.gemv_routed(w["edn"], ids, O.gated_gelu(gu, s.ffn), 1, THREADS)
    assert same_bits(pre.moe["experts_out"].download()[:m], eo)
    assert same_bits(pre.x.download()[:m], O.combine_ranks_add(x1, ws, eo).reshape(m, d))
    # The decode step from each prompt's last token, from the caches prefill left.
    kc, vc = MC.host_caches(eng)
    last = np.array([p[-1] for p in prompts], np.uint32)
    lpos = np.array([n - 1 for n in lens], np.uint32)
    slots = np.arange(batch, dtype=np.uint32)
    eng.set_rows(last, lpos, slots)
    got_ids = eng.step()
    want_ids, want_logits, _ = MC.oracle_decode(eng, layers, embed, final_norm, kc, vc, last, lpos, slots)
    assert same_bits(eng.logits.download(), want_logits)
    assert np.array_equal(got_ids, want_ids)
    pre.close()
