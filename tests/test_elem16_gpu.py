"""Parity of the 16-bit forms of the kernels on a B200, through the C ABI:
bf16 and f16 weights (`*_wbf16`, `*_wf16`) and bf16 and f16 KV caches
(`*_kvbf16`, `*_kvf16`).

A 16-bit weight widens exactly to f32 and a 16-bit cache holds each stored
value rounded to its type (src/FuryKernel/Program/Eval.hs:9), so every form
is held bit for bit to the f32 kernel over the widened weights or caches --
itself bit-exact with the oracle -- and to the oracle directly; the decode
step of a 16-bit model to the oracle's decode over the widened model."""

import math

import numpy as np
import pytest

from furykernel_b200.target import CACHE_SUFFIX, WEIGHT_SUFFIX
from oracle import oracle as O
from tests import model_check as MC

pytestmark = pytest.mark.gpu
TYPES = ("bf16", "f16")

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


def elem16(t, seed, shape, mu=0.0, sigma=0.02):
    """Seeded normals rounded to type t: (bits, the widened values)."""
    bits = MC.narrow(t, O.normal(seed, int(np.prod(shape)), mu, sigma)).reshape(shape)
    return bits, MC.widen(t, bits).reshape(shape)


@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("n,k,m,split", [(11008, 4096, 1, 1), (4096, 11008, 1, 2), (1000, 2048, 3, 4),
                                         (1002, 2048, 4, 1), (300, 1024, 5, 1), (257, 4096, 16, 2),
                                         (1001, 1000, 33, 1), (64, 256, 64, 8)])
def test_gemv_w16_forms(ctx, t, n, k, m, split):
    ws = WEIGHT_SUFFIX[t]
    wbits, w = elem16(t, 61, (n, k))
    x = O.normal(62, m * k).reshape(m, k)
    gbits, g = elem16(t, 63, (k,), 1.0, 0.25)
    r = O.normal(64, m * n).reshape(m, n)
    gu = O.normal(65, m * 2 * k).reshape(m, 2 * k)
    wd, xd, gd, rd, gud = (ctx.to_device(a) for a in (wbits, x, gbits, r, gu))
    yd = ctx.empty((m, n))
    base = {"n": n, "k": k, "m": m, "split": split, "ldx": k, "ldy": n}
    ctx.launch("gemv" + ws, base, [wd, xd, yd])
    assert same_bits(yd.download(), O.gemv(w, x, split, THREADS))
    ctx.launch("gemv_rmsnorm" + ws, dict(base, eps=1e-5, factor=1.0), [wd, xd, gd, yd])
    normed = O.rmsnorm_rows(x, g, 1e-5)
    assert same_bits(yd.download(), O.gemv(w, normed, split, THREADS))
    ctx.launch("gemv_add" + ws, dict(base, ldr=n), [wd, xd, rd, yd])
    assert same_bits(yd.download(), O.add(r, O.gemv(w, x, split, THREADS)))
    act = O.silu_mul(gu[:, :k], gu[:, k:])
    ctx.launch("gemv_silu" + ws, dict(base, ldx=2 * k, up_off=k), [wd, gud, yd])
    assert same_bits(yd.download(), O.gemv(w, act, split, THREADS))
    ctx.launch("gemv_silu_add" + ws, dict(base, ldx=2 * k, ldr=n, up_off=k), [wd, gud, rd, yd])
    assert same_bits(yd.download(), O.add(r, O.gemv(w, act, split, THREADS)))
    if n % 2 == 0 and (m <= 4 or split == 1):  # the SiLU-gate of interleaved gate/up rows (streaming, batched)
        ad = ctx.empty((m, n // 2))
        ctx.launch("gemv_rmsnorm_silu" + ws, dict(base, ldy=n // 2, eps=1e-5, factor=1.0), [wd, xd, gd, ad])
        want = O.silu_mul(O.gemv(np.ascontiguousarray(w[0::2]), normed, split, THREADS),
                          O.gemv(np.ascontiguousarray(w[1::2]), normed, split, THREADS))
        assert same_bits(ad.download(), want)
        ad.free()
    for b in (wd, xd, gd, rd, gud, yd):
        b.free()


@pytest.mark.parametrize("t", TYPES)
def test_gather_rmsnorm_rows_and_split_w16(ctx, t):
    ws = WEIGHT_SUFFIX[t]
    vocab, d, m = 500, 1024, 7
    tbits, table = elem16(t, 71, (vocab, d))
    tok = np.array([3, 499, 0, 17, 17, 250, 1], np.uint32)
    td, tokd, yd = ctx.to_device(tbits), ctx.to_device(tok), ctx.empty((m, d))
    ctx.launch("gather" + ws, {"width": d, "m": m, "factor": 1.0}, [td, tokd, yd])
    assert same_bits(yd.download(), O.gather(table, tok))
    gbits, g = elem16(t, 72, (d,), 1.0, 0.25)
    x = O.normal(73, m * d).reshape(m, d)
    xd, gd, od = ctx.to_device(x), ctx.to_device(gbits), ctx.empty((m, d))
    ctx.launch("rmsnorm_rows" + ws, {"rows": m, "h": d, "eps": 1e-5, "factor": 1.0}, [xd, gd, od])
    assert same_bits(od.download(), O.rmsnorm_rows(x, g, 1e-5))
    hi, lo = ctx.empty(vocab * d), ctx.empty(vocab * d)
    ctx.launch("split_tf32" + ws, {"n": vocab * d}, [td, hi, lo])
    assert same_bits(hi.download(), table.reshape(-1))
    assert not np.any(lo.download().view(np.uint32))
    for b in (td, tokd, yd, xd, gd, od, hi, lo):
        b.free()


@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("m,heads,kv_heads,length,positions,chunk", [
    (2, 4, 2, 64, [5, 40], 16),
    (3, 8, 8, 300, [0, 129, 299], 64),
    (1, 32, 32, 2304, [2048], 128),
    (4, 4, 4, 40, [45, 3, 39, 80], 32),  # positions past the ring's length wrap
    (2, 12, 6, 64, [10, 50], 16),  # the store's 4 heads a block: the second block half idle
])
def test_attention_kv16(ctx, t, m, heads, kv_heads, length, positions, chunk):
    cs = CACHE_SUFFIX[t]
    d = 128
    width = (heads + 2 * kv_heads) * d
    qkv = O.normal(81, m * width).reshape(m, width)
    pos = np.array(positions, np.uint32)
    slot = np.arange(m, dtype=np.uint32)[::-1].copy()
    shape = (m, kv_heads, length, d)
    kbits, kc = elem16(t, 82, shape, 0.0, 1.0)
    vbits, vc = elem16(t, 83, shape, 0.0, 1.0)
    maxpos = int(pos.max()) + 1
    cos_t, sin_t = O.rope_tables(10000.0, d, d // 2, maxpos)
    max_splits = (maxpos + chunk - 1) // chunk
    dq, dkc, dvc, dpos, dslot = (ctx.to_device(a) for a in (qkv, kbits, vbits, pos, slot))
    dcos, dsin = ctx.rope_tables(10000.0, d, d // 2, maxpos)
    pm, pl = ctx.empty(m * heads * max_splits), ctx.empty(m * heads * max_splits)
    pa = ctx.empty(m * heads * max_splits * d)
    out = ctx.empty((m, heads * d))
    store = {"m": m, "kv_heads": kv_heads, "d": d, "length": length, "rotated": d // 2, "ldq": width,
             "k_off": heads * d, "v_off": (heads + kv_heads) * d}
    att = {"m": m, "heads": heads, "kv_heads": kv_heads, "d": d, "length": length, "rotated": d // 2,
           "chunk": chunk, "max_splits": max_splits, "ldq": width, "q_off": 0, "scale": 1.0 / math.sqrt(d)}
    comb = {"m": m, "heads": heads, "d": d, "chunk": chunk, "max_splits": max_splits, "ldo": heads * d}
    ctx.launch("kv_store_ring" + cs, store, [dq, dcos, dsin, dpos, dslot, dkc, dvc])
    ctx.launch("attend_split" + cs, att, [dq, dcos, dsin, dpos, dslot, dkc, dvc, pm, pl, pa])
    ctx.launch("attend_combine", comb, [pm, pl, pa, dpos, out])

    # The oracle: the stores rounded to the cache's type, the attention over the caches as held.
    kcache, vcache = kc.copy(), vc.copy()
    krot = O.rope(qkv[:, heads * d:(heads + kv_heads) * d], kv_heads, d, d // 2, pos, cos_t, sin_t)
    vnew = np.ascontiguousarray(qkv[:, (heads + kv_heads) * d:])
    O.kv_store_ring(MC.rounded(t, krot), kv_heads, d, length, pos, slot, kcache)
    O.kv_store_ring(MC.rounded(t, vnew), kv_heads, d, length, pos, slot, vcache)
    assert np.array_equal(dkc.download(), MC.narrow(t, kcache).reshape(shape))
    assert np.array_equal(dvc.download(), MC.narrow(t, vcache).reshape(shape))
    qrot = O.rope(qkv[:, :heads * d], heads, d, d // 2, pos, cos_t, sin_t)
    want, _ = O.attend(qrot, heads, kv_heads, d, length, pos, slot, kcache, vcache,
                       np.float32(1.0 / math.sqrt(d)), chunk, 4, max_splits, THREADS)
    assert same_bits(out.download(), want)
    # The fused decode form: the same bits, the same caches.
    dkc.upload(kbits)
    dvc.upload(vbits)
    ctx.launch("attend_decode" + cs, dict(att, k_off=heads * d, v_off=(heads + kv_heads) * d),
               [dq, dcos, dsin, dpos, dslot, dkc, dvc, pm, pl, pa])
    ctx.launch("attend_combine", comb, [pm, pl, pa, dpos, out])
    assert same_bits(out.download(), want)
    assert np.array_equal(dkc.download(), MC.narrow(t, kcache).reshape(shape))
    assert np.array_equal(dvc.download(), MC.narrow(t, vcache).reshape(shape))
    for b in (dq, dkc, dvc, dpos, dslot, dcos, dsin, pm, pl, pa, out):
        b.free()


@pytest.mark.parametrize("t", TYPES)
def test_attend_prompt_kv16_matches_the_f32_form_over_widened_caches(ctx, t):
    """The prompt attention (prefill) reads the 16-bit caches widened: the
    f32 form over the widened caches gives the same bits."""
    m, heads, kv_heads, d, length = 70, 4, 2, 128, 128
    width = (heads + 2 * kv_heads) * d
    qkv = O.normal(91, m * width).reshape(m, width)
    pos = np.arange(m, dtype=np.uint32)
    slot = np.zeros(m, np.uint32)
    shape = (1, kv_heads, length, d)
    kbits, kc = elem16(t, 92, shape, 0.0, 1.0)
    vbits, vc = elem16(t, 93, shape, 0.0, 1.0)
    dq, dpos, dslot = ctx.to_device(qkv), ctx.to_device(pos), ctx.to_device(slot)
    dcos, dsin = ctx.rope_tables(10000.0, d, d // 2, length)
    k16, v16, k32, v32 = (ctx.to_device(a) for a in (kbits, vbits, kc, vc))
    o16, o32 = ctx.empty((m, heads * d)), ctx.empty((m, heads * d))
    p = {"m": m, "heads": heads, "kv_heads": kv_heads, "d": d, "length": length, "rotated": d // 2, "ldq": width,
         "q_off": 0, "ldo": heads * d, "max_pos": m - 1, "scale": 1.0 / math.sqrt(d)}
    ctx.launch("attend_prompt" + CACHE_SUFFIX[t], p, [dq, dcos, dsin, dpos, dslot, k16, v16, o16])
    ctx.launch("attend_prompt", p, [dq, dcos, dsin, dpos, dslot, k32, v32, o32])
    assert same_bits(o16.download(), o32.download())
    for b in (dq, dpos, dslot, dcos, dsin, k16, v16, k32, v32, o16, o32):
        b.free()


def small_shape(batch, weights="bf16", cache="bf16"):
    from furykernel_b200.shape import LlamaShape

    return LlamaShape(d_model=512, heads=4, kv_heads=4, head_dim=128, ffn=1024, vocab=3000, layers=2, slots=batch,
                      length=96, positions=96, weights=weights, cache=cache)


@pytest.mark.parametrize("batch,fused,weights,cache", [(1, None, "bf16", "bf16"), (3, False, "bf16", "bf16"),
                                                       (4, None, "bf16", "bf16"), (9, None, "bf16", "bf16"),
                                                       (2, None, "bf16", "f32"), (5, None, "f32", "bf16"),
                                                       (1, None, "f16", "f16"), (3, False, "f16", "f16"),
                                                       (9, None, "f16", "f16"), (2, None, "f16", "bf16"),
                                                       (5, None, "bf16", "f16")])
def test_w16_model_decode_step(ctx, batch, fused, weights, cache):
    """A decode step of a model with 16-bit weights and/or caches, captured
    as a graph, against the oracle's decode over the widened model: the
    same ids, logits and residual rows, bit for bit, and the same caches."""
    from furykernel_b200.engine import Llama

    s = small_shape(batch, weights, cache)
    eng = Llama(ctx, s, batch, seed=300 + batch, chunk=32, prefill_kv=1.0, fuse_attention=fused)
    tokens = O.ints(9 + batch, batch, s.vocab)
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
    gk, gv = MC.host_caches(eng)
    assert same_bits(gk, kc) and same_bits(gv, vc)


@pytest.mark.parametrize("t", TYPES)
def test_stores_round_the_edge_values_as_the_reference_narrows_them(ctx, t):
    """A value row through the KV store (values are stored as they come):
    the largest finite values, the ties just short of and at overflow, the
    smallest subnormals and their ties, signed zeros, NaNs and infinities
    narrow as narrowBF16 / narrowF16 do (Numerics.hs:41-48, :100-130)."""
    d, kv_heads = 128, 1
    edge = np.array([65504, 65519.996, 65520, 2.0 ** -24, 2.0 ** -25, 1.5 * 2.0 ** -24, -0.0, 1e-30, -1e6,
                     3.4e38, 1 + 2.0 ** -11, 1 + 3 * 2.0 ** -11, 1 + 2.0 ** -8, 1 + 3 * 2.0 ** -8], np.float32)
    specials = np.array([0xFF800001, 0x7FC00000, 0x7F800000, 0xFF800000, 0x00000001, 0x80400000], np.uint32)
    v = np.concatenate([edge, specials.view(np.float32)])
    v = np.concatenate([v, O.normal(95, d - v.size)]).astype(np.float32)
    qkv = np.concatenate([O.normal(96, 2 * d), v]).reshape(1, 3 * d).astype(np.float32)
    pos, slot = np.zeros(1, np.uint32), np.zeros(1, np.uint32)
    dq, dpos, dslot = ctx.to_device(qkv), ctx.to_device(pos), ctx.to_device(slot)
    dcos, dsin = ctx.rope_tables(10000.0, d, d // 2, 1)
    dk, dv = ctx.zeros(d, np.uint16), ctx.zeros(d, np.uint16)
    ctx.launch("kv_store_ring" + CACHE_SUFFIX[t],
               {"m": 1, "kv_heads": kv_heads, "d": d, "length": 1, "rotated": d // 2, "ldq": 3 * d, "k_off": d,
                "v_off": 2 * d}, [dq, dcos, dsin, dpos, dslot, dk, dv])
    assert np.array_equal(dv.download(), MC.narrow(t, v))
    for b in (dq, dpos, dslot, dcos, dsin, dk, dv):
        b.free()


def test_fill_normal_f16_is_the_f32_fill_rounded(ctx):
    n = 1 << 16
    a, h = ctx.empty(n), ctx.zeros(n, np.uint16)
    ctx.fill_normal(a, 123, 0.0, 0.02)
    ctx.fill_normal_f16(h, 123, 0.0, 0.02)
    assert np.array_equal(h.download(), O.narrow_f16(a.download()))
    a.free()
    h.free()


@pytest.mark.parametrize("weights,cache,one_slot", [("bf16", "bf16", False), ("f16", "f16", False),
                                                    ("f16", "f16", True), ("bf16", "f16", True)])
def test_w16_prefill_then_decode(ctx, weights, cache, one_slot):
    """Prefill of 16-bit models: the caches it leaves hold what the
    reference's evaluator allows a store of each element in the cache's
    type (mayStore, Eval.hs:924-944); the decode step from them is the
    oracle's bit for bit; the last rows' logits lie within the evaluator's
    bounds."""
    from furykernel_b200.engine import Llama
    from furykernel_b200.prefill import Prefill, prompt_chunks

    batch = 2
    s = small_shape(batch, weights, cache)
    eng = Llama(ctx, s, batch, seed=350, chunk=16)
    pre = Prefill(eng, rows=128, one_slot=one_slot)
    layers, embed, final_norm = MC.host_model(eng)
    lens = [40, 23]
    prompts = [O.ints(180 + i, n, s.vocab) for i, n in enumerate(lens)]
    slots = np.arange(batch, dtype=np.uint32)
    toks = np.concatenate([p[:-1] for p in prompts])
    poss = np.concatenate([np.arange(n - 1, dtype=np.uint32) for n in lens])
    sl = np.concatenate([np.full(n - 1, i, np.uint32) for i, n in enumerate(lens)])
    for i, n in prompt_chunks(pre, toks, poss, sl):
        pre.run(toks[i:i + n], poss[i:i + n], sl[i:i + n])
    ctx.sync()
    kc_p, vc_p = MC.host_caches(eng)
    _, _, stored_ok = MC.referee_decode(eng, layers, embed, final_norm, kc_p, vc_p, toks, poss, sl)
    assert stored_ok
    last = np.array([p[-1] for p in prompts], np.uint32)
    lpos = np.array([n - 1 for n in lens], np.uint32)
    eng.set_rows(last, lpos, slots)
    ids = eng.step()
    want_ids, want_logits, _ = MC.oracle_decode(eng, layers, embed, final_norm, kc_p.copy(), vc_p.copy(), last,
                                                lpos, slots)
    assert same_bits(eng.logits.download(), want_logits)
    assert np.array_equal(ids, want_ids)
    pre.close()
