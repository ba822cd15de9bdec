"""Parity of the bf16 forms of the kernels (bf16 weights `*_wbf16`, bf16 KV
caches `*_kvbf16`) on a B200, through the C ABI.

A bf16 weight widens exactly to f32 and a bf16 cache holds each stored
value rounded to bf16 (src/FuryKernel/Program/Eval.hs:9), so every form is
held bit for bit to the f32 kernel over the widened weights or caches --
itself bit-exact with the oracle -- and to the oracle directly; the decode
step of a bf16 model to the oracle's decode over the widened model.

These forms have not run on a B200 yet: the module runs only with
FURYKERNEL_NEW_KERNELS=1 in the environment, so that a run of the GPU suite
exercises only kernels that have passed on a GPU before."""

import math
import os

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(os.environ.get("FURYKERNEL_NEW_KERNELS") != "1",
                                 reason="the bf16 forms have not run on a B200 yet (FURYKERNEL_NEW_KERNELS=1 runs them)")]

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


def bf16(seed, shape, mu=0.0, sigma=0.02):
    """Seeded normals rounded to bf16: (bits, the widened values)."""
    bits = O.narrow_bf16(O.normal(seed, int(np.prod(shape)), mu, sigma)).reshape(shape)
    return bits, O.widen_bf16(bits).reshape(shape)


@pytest.mark.parametrize("n,k,m,split", [(11008, 4096, 1, 1), (4096, 11008, 1, 2), (1000, 2048, 3, 4),
                                         (1002, 2048, 4, 1), (300, 1024, 5, 1), (257, 4096, 16, 2),
                                         (1001, 1000, 33, 1), (64, 256, 64, 8)])
def test_gemv_wbf16_forms(ctx, n, k, m, split):
    wbits, w = bf16(61, (n, k))
    x = O.normal(62, m * k).reshape(m, k)
    gbits, g = bf16(63, (k,), 1.0, 0.25)
    r = O.normal(64, m * n).reshape(m, n)
    gu = O.normal(65, m * 2 * k).reshape(m, 2 * k)
    wd, xd, gd, rd, gud = (ctx.to_device(a) for a in (wbits, x, gbits, r, gu))
    yd = ctx.empty((m, n))
    base = {"n": n, "k": k, "m": m, "split": split, "ldx": k, "ldy": n}
    ctx.launch("gemv_wbf16", base, [wd, xd, yd])
    assert same_bits(yd.download(), O.gemv(w, x, split, THREADS))
    ctx.launch("gemv_rmsnorm_wbf16", dict(base, eps=1e-5, factor=1.0), [wd, xd, gd, yd])
    normed = O.rmsnorm_rows(x, g, 1e-5)
    assert same_bits(yd.download(), O.gemv(w, normed, split, THREADS))
    ctx.launch("gemv_add_wbf16", dict(base, ldr=n), [wd, xd, rd, yd])
    assert same_bits(yd.download(), O.add(r, O.gemv(w, x, split, THREADS)))
    act = O.silu_mul(gu[:, :k], gu[:, k:])
    ctx.launch("gemv_silu_wbf16", dict(base, ldx=2 * k, up_off=k), [wd, gud, yd])
    assert same_bits(yd.download(), O.gemv(w, act, split, THREADS))
    ctx.launch("gemv_silu_add_wbf16", dict(base, ldx=2 * k, ldr=n, up_off=k), [wd, gud, rd, yd])
    assert same_bits(yd.download(), O.add(r, O.gemv(w, act, split, THREADS)))
    if n % 2 == 0 and (m <= 4 or split == 1):  # the SiLU-gate of interleaved gate/up rows (streaming, batched)
        ad = ctx.empty((m, n // 2))
        ctx.launch("gemv_rmsnorm_silu_wbf16", dict(base, ldy=n // 2, eps=1e-5, factor=1.0), [wd, xd, gd, ad])
        want = O.silu_mul(O.gemv(np.ascontiguousarray(w[0::2]), normed, split, THREADS),
                          O.gemv(np.ascontiguousarray(w[1::2]), normed, split, THREADS))
        assert same_bits(ad.download(), want)
        ad.free()
    for b in (wd, xd, gd, rd, gud, yd):
        b.free()


def test_gather_rmsnorm_rows_and_split_wbf16(ctx):
    vocab, d, m = 500, 1024, 7
    tbits, table = bf16(71, (vocab, d))
    tok = np.array([3, 499, 0, 17, 17, 250, 1], np.uint32)
    td, tokd, yd = ctx.to_device(tbits), ctx.to_device(tok), ctx.empty((m, d))
    ctx.launch("gather_wbf16", {"width": d, "m": m, "factor": 1.0}, [td, tokd, yd])
    assert same_bits(yd.download(), O.gather(table, tok))
    gbits, g = bf16(72, (d,), 1.0, 0.25)
    x = O.normal(73, m * d).reshape(m, d)
    xd, gd, od = ctx.to_device(x), ctx.to_device(gbits), ctx.empty((m, d))
    ctx.launch("rmsnorm_rows_wbf16", {"rows": m, "h": d, "eps": 1e-5, "factor": 1.0}, [xd, gd, od])
    assert same_bits(od.download(), O.rmsnorm_rows(x, g, 1e-5))
    hi, lo = ctx.empty(vocab * d), ctx.empty(vocab * d)
    ctx.launch("split_tf32_wbf16", {"n": vocab * d}, [td, hi, lo])
    assert same_bits(hi.download(), table.reshape(-1))
    assert not np.any(lo.download().view(np.uint32))
    for b in (td, tokd, yd, xd, gd, od, hi, lo):
        b.free()


@pytest.mark.parametrize("m,heads,kv_heads,length,positions,chunk", [
    (2, 4, 2, 64, [5, 40], 16),
    (3, 8, 8, 300, [0, 129, 299], 64),
    (1, 32, 32, 2304, [2048], 128),
    (4, 4, 4, 40, [45, 3, 39, 80], 32),  # positions past the ring's length wrap
])
def test_attention_kvbf16(ctx, m, heads, kv_heads, length, positions, chunk):
    d = 128
    width = (heads + 2 * kv_heads) * d
    qkv = O.normal(81, m * width).reshape(m, width)
    pos = np.array(positions, np.uint32)
    slot = np.arange(m, dtype=np.uint32)[::-1].copy()
    shape = (m, kv_heads, length, d)
    kbits, kc = bf16(82, shape, 0.0, 1.0)
    vbits, vc = bf16(83, shape, 0.0, 1.0)
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
    ctx.launch("kv_store_ring_kvbf16", store, [dq, dcos, dsin, dpos, dslot, dkc, dvc])
    ctx.launch("attend_split_kvbf16", att, [dq, dcos, dsin, dpos, dslot, dkc, dvc, pm, pl, pa])
    ctx.launch("attend_combine", comb, [pm, pl, pa, dpos, out])

    # The oracle: the stores rounded to bf16, the attention over the caches as held.
    kcache, vcache = kc.copy(), vc.copy()
    krot = O.rope(qkv[:, heads * d:(heads + kv_heads) * d], kv_heads, d, d // 2, pos, cos_t, sin_t)
    vnew = np.ascontiguousarray(qkv[:, (heads + kv_heads) * d:])
    O.kv_store_ring(O.widen_bf16(O.narrow_bf16(krot)).reshape(krot.shape), kv_heads, d, length, pos, slot, kcache)
    O.kv_store_ring(O.widen_bf16(O.narrow_bf16(vnew)).reshape(vnew.shape), kv_heads, d, length, pos, slot, vcache)
    assert np.array_equal(dkc.download(), O.narrow_bf16(kcache).reshape(shape))
    assert np.array_equal(dvc.download(), O.narrow_bf16(vcache).reshape(shape))
    qrot = O.rope(qkv[:, :heads * d], heads, d, d // 2, pos, cos_t, sin_t)
    want, _ = O.attend(qrot, heads, kv_heads, d, length, pos, slot, kcache, vcache,
                       np.float32(1.0 / math.sqrt(d)), chunk, 4, max_splits, THREADS)
    assert same_bits(out.download(), want)
    # The fused decode form: the same bits, the same caches.
    dkc.upload(kbits)
    dvc.upload(vbits)
    ctx.launch("attend_decode_kvbf16", dict(att, k_off=heads * d, v_off=(heads + kv_heads) * d),
               [dq, dcos, dsin, dpos, dslot, dkc, dvc, pm, pl, pa])
    ctx.launch("attend_combine", comb, [pm, pl, pa, dpos, out])
    assert same_bits(out.download(), want)
    assert np.array_equal(dkc.download(), O.narrow_bf16(kcache).reshape(shape))
    assert np.array_equal(dvc.download(), O.narrow_bf16(vcache).reshape(shape))
    for b in (dq, dkc, dvc, dpos, dslot, dcos, dsin, pm, pl, pa, out):
        b.free()


def test_attend_prompt_kvbf16_matches_the_f32_form_over_widened_caches(ctx):
    """The prompt attention (prefill) reads the bf16 caches widened: the f32
    form over the widened caches gives the same bits."""
    m, heads, kv_heads, d, length = 70, 4, 2, 128, 128
    width = (heads + 2 * kv_heads) * d
    qkv = O.normal(91, m * width).reshape(m, width)
    pos = np.arange(m, dtype=np.uint32)
    slot = np.zeros(m, np.uint32)
    shape = (1, kv_heads, length, d)
    kbits, kc = bf16(92, shape, 0.0, 1.0)
    vbits, vc = bf16(93, shape, 0.0, 1.0)
    dq, dpos, dslot = ctx.to_device(qkv), ctx.to_device(pos), ctx.to_device(slot)
    dcos, dsin = ctx.rope_tables(10000.0, d, d // 2, length)
    k16, v16, k32, v32 = (ctx.to_device(a) for a in (kbits, vbits, kc, vc))
    o16, o32 = ctx.empty((m, heads * d)), ctx.empty((m, heads * d))
    p = {"m": m, "heads": heads, "kv_heads": kv_heads, "d": d, "length": length, "rotated": d // 2, "ldq": width,
         "q_off": 0, "ldo": heads * d, "max_pos": m - 1, "scale": 1.0 / math.sqrt(d)}
    ctx.launch("attend_prompt_kvbf16", p, [dq, dcos, dsin, dpos, dslot, k16, v16, o16])
    ctx.launch("attend_prompt", p, [dq, dcos, dsin, dpos, dslot, k32, v32, o32])
    assert same_bits(o16.download(), o32.download())
    for b in (dq, dpos, dslot, dcos, dsin, k16, v16, k32, v32, o16, o32):
        b.free()


def small_shape(batch, weights="bf16", cache="bf16"):
    from furykernel_b200.program.llama import LlamaShape

    return LlamaShape(d_model=512, heads=4, kv_heads=4, head_dim=128, ffn=1024, vocab=3000, layers=2, slots=batch,
                      length=96, positions=96, weights=weights, cache=cache)


@pytest.mark.parametrize("batch,fused,weights,cache", [(1, None, "bf16", "bf16"), (3, False, "bf16", "bf16"),
                                                       (4, None, "bf16", "bf16"), (9, None, "bf16", "bf16"),
                                                       (2, None, "bf16", "f32"), (5, None, "f32", "bf16")])
def test_bf16_model_decode_step(ctx, batch, fused, weights, cache):
    """A decode step of a model with bf16 weights and/or caches, captured
    as a graph, against the oracle's decode over the widened model: the
    same ids, logits and residual rows, bit for bit, and the same caches."""
    from furykernel_b200.engine import Llama
    from tests import model_check as MC

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
