"""Parity of the paged-cache kernels (`*_paged`, f32, bf16 and f16 caches)
on a B200, through the C ABI.

A paged cache holds a row's position t in block table[t / block_size] of a
pool (src/FuryKernel/Program/Eval.hs:592-602); the kernels keep the ring
kernels' arithmetic position for position, so each is held bit for bit to
the oracle's ring arithmetic over the row's blocks gathered in table order
(tests/model_check.py: pool_to_rings), and the decode step of a model with
paged caches to the oracle's decode."""

import math

import numpy as np
import pytest

from furykernel_b200.target import CACHE_SUFFIX
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


def block_addresses(ctx, pool, blocks):
    """A pool's blocks as a table of their device addresses (u64), as the
    kernels' k_cache / v_cache tables bind them."""
    per = pool.nbytes // blocks
    return ctx.to_device(np.uint64(pool.ptr) + np.arange(blocks, dtype=np.uint64) * np.uint64(per))


def disjoint_tables(seed, m, table_len, blocks):
    """Each row its own blocks, in a shuffled order."""
    perm = np.random.default_rng(seed).permutation(blocks)[:m * table_len]
    return perm.reshape(m, table_len).astype(np.uint32)


@pytest.mark.parametrize("t", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("m,heads,kv_heads,block_size,positions,chunk", [
    (2, 4, 2, 16, [5, 40], 16),
    (3, 8, 8, 32, [0, 129, 191], 64),
    (1, 32, 32, 16, [2047], 128),
    (2, 12, 6, 16, [10, 50], 16),  # the store's 4 heads a block: the second block half idle
])
def test_paged_store_and_attention(ctx, t, m, heads, kv_heads, block_size, positions, chunk):
    d = 128
    width = (heads + 2 * kv_heads) * d
    qkv = O.normal(101, m * width).reshape(m, width)
    pos = np.array(positions, np.uint32)
    span = int(pos.max()) + 1
    table_len = (span + block_size - 1) // block_size
    blocks = m * table_len + 3
    tables = disjoint_tables(102, m, table_len, blocks)
    shape = (blocks, kv_heads, block_size, d)
    kpool = O.normal(103, int(np.prod(shape))).reshape(shape)
    vpool = O.normal(104, int(np.prod(shape))).reshape(shape)
    if t != "f32":
        kbits, vbits = MC.narrow(t, kpool).reshape(shape), MC.narrow(t, vpool).reshape(shape)
        kpool, vpool = MC.widen(t, kbits).reshape(shape), MC.widen(t, vbits).reshape(shape)
        dk, dv = ctx.to_device(kbits), ctx.to_device(vbits)
    else:
        dk, dv = ctx.to_device(kpool), ctx.to_device(vpool)
    cos_t, sin_t = O.rope_tables(10000.0, d, d // 2, span)
    max_splits = (span + chunk - 1) // chunk
    dq, dpos, dtab = ctx.to_device(qkv), ctx.to_device(pos), ctx.to_device(tables)
    dcos, dsin = ctx.rope_tables(10000.0, d, d // 2, span)
    pm, pl = ctx.empty(m * heads * max_splits), ctx.empty(m * heads * max_splits)
    pa = ctx.empty(m * heads * max_splits * d)
    out = ctx.empty((m, heads * d))
    suffix = CACHE_SUFFIX[t]
    pg = {"block_size": block_size, "table_len": table_len, "blocks": blocks}
    dkt, dvt = block_addresses(ctx, dk, blocks), block_addresses(ctx, dv, blocks)
    ctx.launch("kv_store_paged" + suffix,
               dict(pg, m=m, kv_heads=kv_heads, d=d, rotated=d // 2, ldq=width, k_off=heads * d,
                    v_off=(heads + kv_heads) * d), [dq, dcos, dsin, dpos, dtab, dkt, dvt])
    ctx.launch("attend_split_paged" + suffix,
               dict(pg, m=m, heads=heads, kv_heads=kv_heads, d=d, rotated=d // 2, chunk=chunk, max_splits=max_splits,
                    ldq=width, q_off=0, scale=1.0 / math.sqrt(d)),
               [dq, dcos, dsin, dpos, dtab, pm, pl, pa, dkt, dvt])
    ctx.launch("attend_combine", {"m": m, "heads": heads, "d": d, "chunk": chunk, "max_splits": max_splits,
                                  "ldo": heads * d}, [pm, pl, pa, dpos, out])

    # The oracle: each row's blocks as a ring, the stores, the ring attention.
    def as_stored(a):
        return MC.rounded(t, a)

    kr, vr = MC.pool_to_rings(kpool, tables), MC.pool_to_rings(vpool, tables)
    length, rows = table_len * block_size, np.arange(m, dtype=np.uint32)
    krot = O.rope(qkv[:, heads * d:(heads + kv_heads) * d], kv_heads, d, d // 2, pos, cos_t, sin_t)
    O.kv_store_ring(as_stored(krot), kv_heads, d, length, pos, rows, kr)
    O.kv_store_ring(as_stored(np.ascontiguousarray(qkv[:, (heads + kv_heads) * d:])), kv_heads, d, length, pos,
                    rows, vr)
    kwant, vwant = kpool.copy(), vpool.copy()
    MC.rings_to_pool(kr, tables, kwant)
    MC.rings_to_pool(vr, tables, vwant)
    if t != "f32":
        assert np.array_equal(dk.download(), MC.narrow(t, kwant).reshape(shape))
        assert np.array_equal(dv.download(), MC.narrow(t, vwant).reshape(shape))
    else:
        assert same_bits(dk.download(), kwant) and same_bits(dv.download(), vwant)
    qrot = O.rope(qkv[:, :heads * d], heads, d, d // 2, pos, cos_t, sin_t)
    want, _ = O.attend(qrot, heads, kv_heads, d, length, pos, rows, kr, vr, np.float32(1.0 / math.sqrt(d)), chunk,
                       4, max_splits, THREADS)
    assert same_bits(out.download(), want)
    # The fused form (the store folded into the attention; the tables'
    # entries distinct): the same output and the same pools.
    dk.upload(kbits if t != "f32" else kpool)
    dv.upload(vbits if t != "f32" else vpool)
    ctx.launch("attend_decode_paged" + suffix,
               dict(pg, m=m, heads=heads, kv_heads=kv_heads, d=d, rotated=d // 2, chunk=chunk, max_splits=max_splits,
                    ldq=width, q_off=0, k_off=heads * d, v_off=(heads + kv_heads) * d, scale=1.0 / math.sqrt(d)),
               [dq, dcos, dsin, dpos, dtab, pm, pl, pa, dkt, dvt])
    ctx.launch("attend_combine", {"m": m, "heads": heads, "d": d, "chunk": chunk, "max_splits": max_splits,
                                  "ldo": heads * d}, [pm, pl, pa, dpos, out])
    assert same_bits(out.download(), want)
    if t != "f32":
        assert np.array_equal(dk.download(), MC.narrow(t, kwant).reshape(shape))
        assert np.array_equal(dv.download(), MC.narrow(t, vwant).reshape(shape))
    else:
        assert same_bits(dk.download(), kwant) and same_bits(dv.download(), vwant)
    for b in (dq, dpos, dtab, dk, dv, dkt, dvt, dcos, dsin, pm, pl, pa, out):
        b.free()


@pytest.mark.parametrize("t", ["f32", "bf16", "f16"])
def test_paged_prompt_attention_matches_the_ring_form(ctx, t):
    """One prompt's rows through its block table: the same bits as the ring
    prompt kernel over the blocks gathered into a slot."""
    m, heads, kv_heads, d, block_size = 70, 4, 2, 128, 16
    width = (heads + 2 * kv_heads) * d
    table_len, blocks = 5, 12
    qkv = O.normal(111, m * width).reshape(m, width)
    pos = np.arange(m, dtype=np.uint32)
    table = disjoint_tables(112, 1, table_len, blocks)
    tables = np.repeat(table, m, axis=0)
    shape = (blocks, kv_heads, block_size, d)
    kpool = O.normal(113, int(np.prod(shape))).reshape(shape)
    vpool = O.normal(114, int(np.prod(shape))).reshape(shape)
    if t != "f32":
        kbits, vbits = MC.narrow(t, kpool).reshape(shape), MC.narrow(t, vpool).reshape(shape)
        kpool, vpool = MC.widen(t, kbits).reshape(shape), MC.widen(t, vbits).reshape(shape)
        dk, dv = ctx.to_device(kbits), ctx.to_device(vbits)
    else:
        dk, dv = ctx.to_device(kpool), ctx.to_device(vpool)
    length = table_len * block_size
    ring_k = MC.pool_to_rings(kpool, table)  # [1, kv_heads, length, d]
    ring_v = MC.pool_to_rings(vpool, table)
    rk, rv = ctx.to_device(ring_k), ctx.to_device(ring_v)
    dq, dpos, dtab, dslot = ctx.to_device(qkv), ctx.to_device(pos), ctx.to_device(tables), ctx.zeros(m, np.uint32)
    dcos, dsin = ctx.rope_tables(10000.0, d, d // 2, length)
    o_paged, o_ring = ctx.empty((m, heads * d)), ctx.empty((m, heads * d))
    common = {"m": m, "heads": heads, "kv_heads": kv_heads, "d": d, "rotated": d // 2, "ldq": width, "q_off": 0,
              "ldo": heads * d, "max_pos": m - 1, "scale": 1.0 / math.sqrt(d)}
    dkt, dvt = block_addresses(ctx, dk, blocks), block_addresses(ctx, dv, blocks)
    ctx.launch("attend_prompt_paged" + CACHE_SUFFIX[t],
               dict(common, block_size=block_size, table_len=table_len, blocks=blocks),
               [dq, dcos, dsin, dpos, dtab, o_paged, dkt, dvt])
    ctx.launch("attend_prompt", dict(common, length=length), [dq, dcos, dsin, dpos, dslot, rk, rv, o_ring])
    assert same_bits(o_paged.download(), o_ring.download())
    for b in (dk, dv, dkt, dvt, rk, rv, dq, dpos, dtab, dslot, dcos, dsin, o_paged, o_ring):
        b.free()


@pytest.mark.parametrize("batch,cache", [(1, "f32"), (3, "f32"), (9, "bf16"), (2, "bf16"), (4, "f16")])
def test_paged_model_decode_step(ctx, batch, cache):
    """A decode step of a model with paged caches, captured as a graph,
    against the oracle's decode over the rows' blocks: the same ids, logits
    and residual rows, bit for bit, and the same pools."""
    from furykernel_b200.engine import Llama
    from furykernel_b200.shape import LlamaShape

    s = LlamaShape(d_model=512, heads=4, kv_heads=4, head_dim=128, ffn=1024, vocab=3000, layers=2, positions=96,
                   blocks=6 * batch + 5, block_size=16, cache=cache)
    eng = Llama(ctx, s, batch, seed=400 + batch, chunk=32, prefill_kv=1.0)
    tokens = O.ints(19 + batch, batch, s.vocab)
    pos = ((np.arange(batch) * 37 + 5) % 96).astype(np.uint32)
    tables = disjoint_tables(120 + batch, batch, s.table_len, s.blocks)
    layers, embed, final_norm = MC.host_model(eng)
    kc, vc = MC.host_caches(eng)
    eng.set_rows(tokens, pos, tables)
    ids = eng.step()
    want_ids, want_logits, want_x = MC.oracle_decode(eng, layers, embed, final_norm, kc, vc, tokens, pos, tables)
    assert np.array_equal(ids, want_ids)
    assert same_bits(eng.logits.download(), want_logits)
    assert same_bits(eng.x.download(), want_x)
    gk, gv = MC.host_caches(eng)
    assert same_bits(gk, kc) and same_bits(gv, vc)


@pytest.mark.parametrize("cache,one_slot", [("f32", False), ("f32", True), ("bf16", True), ("f16", False)])
def test_paged_prefill_then_decode(ctx, cache, one_slot):
    """Prompts prefilled into a paged pool through the rows' block tables,
    then a decode step (fused: the tables' entries distinct) from the pools
    prefill left: the oracle's ids and logits, bit for bit."""
    from furykernel_b200.engine import Llama
    from furykernel_b200.prefill import Prefill, prompt_chunks
    from furykernel_b200.shape import LlamaShape

    batch = 2
    s = LlamaShape(d_model=512, heads=4, kv_heads=4, head_dim=128, ffn=1024, vocab=3000, layers=2, positions=96,
                   blocks=2 * 6 + 4, block_size=16, cache=cache)
    eng = Llama(ctx, s, batch, seed=620, chunk=16)
    pre = Prefill(eng, rows=128, one_slot=one_slot)
    layers, embed, final_norm = MC.host_model(eng)
    tables = disjoint_tables(621, batch, s.table_len, s.blocks)
    lens = [37, 52]
    prompts = [O.ints(640 + i, n, s.vocab) for i, n in enumerate(lens)]
    toks = np.concatenate([p[:-1] for p in prompts])
    poss = np.concatenate([np.arange(n - 1, dtype=np.uint32) for n in lens])
    rows = np.concatenate([np.full(n - 1, i) for i, n in enumerate(lens)])
    for i, n in prompt_chunks(pre, toks, poss, rows):
        pre.run(toks[i:i + n], poss[i:i + n], tables[rows[i:i + n]])
    ctx.sync()
    kc, vc = MC.host_caches(eng)
    last = np.array([p[-1] for p in prompts], np.uint32)
    lpos = np.array([n - 1 for n in lens], np.uint32)
    eng.set_rows(last, lpos, tables)
    ids = eng.step()
    want_ids, want_logits, _ = MC.oracle_decode(eng, layers, embed, final_norm, kc, vc, last, lpos, tables)
    assert same_bits(eng.logits.download(), want_logits)
    assert np.array_equal(ids, want_ids)
    pre.close()


def scattered_blocks(ctx, pool_bits, seed):
    """Every block of a host pool [blocks, ...] copied into an allocation of
    its own, the allocations made in a shuffled order with spacers between
    them (so that no two blocks are adjacent or in pool order). Returns the
    allocations by block and everything to free."""
    blocks = pool_bits.shape[0]
    order = np.random.default_rng(seed).permutation(blocks)
    by_block, keep = [None] * blocks, []
    for b in order:
        keep.append(ctx.empty(4096 // 4))  # a spacer
        buf = ctx.to_device(np.ascontiguousarray(pool_bits[b]))
        by_block[b] = buf
        keep.append(buf)
    return by_block, keep


def gathered(bufs, shape, dtype):
    """The blocks' allocations read back as one pool array."""
    return np.stack([b.download().view(dtype).reshape(shape[1:]) for b in bufs])


@pytest.mark.parametrize("t", ["f32", "bf16"])
def test_paged_blocks_allocated_apart(ctx, t):
    """The reference's paged layout (Graph.hs:144-152): each block an array
    of its own wherever it was allocated, reached through the caches' tables
    of block addresses. Blocks allocated one by one, out of order and apart:
    the store, the split attention and the fused decode attention give the
    oracle's bits, and each block holds what the oracle stored there."""
    m, heads, kv_heads, d, block_size, chunk = 3, 8, 4, 128, 16, 32
    width = (heads + 2 * kv_heads) * d
    pos = np.array([3, 70, 45], np.uint32)
    span = int(pos.max()) + 1
    table_len = (span + block_size - 1) // block_size
    blocks = m * table_len + 2
    tables = disjoint_tables(131, m, table_len, blocks)
    shape = (blocks, kv_heads, block_size, d)
    qkv = O.normal(132, m * width).reshape(m, width)
    kpool = O.normal(133, int(np.prod(shape))).reshape(shape)
    vpool = O.normal(134, int(np.prod(shape))).reshape(shape)
    if t != "f32":
        kbits, vbits = MC.narrow(t, kpool).reshape(shape), MC.narrow(t, vpool).reshape(shape)
        kpool, vpool = MC.widen(t, kbits).reshape(shape), MC.widen(t, vbits).reshape(shape)
        dtype = np.uint16
    else:
        kbits, vbits, dtype = kpool, vpool, np.float32
    suffix = CACHE_SUFFIX[t]
    pg = {"block_size": block_size, "table_len": table_len, "blocks": blocks}
    cos_t, sin_t = O.rope_tables(10000.0, d, d // 2, span)
    max_splits = (span + chunk - 1) // chunk
    dq, dpos, dtab = ctx.to_device(qkv), ctx.to_device(pos), ctx.to_device(tables)
    dcos, dsin = ctx.rope_tables(10000.0, d, d // 2, span)
    pm, pl = ctx.empty(m * heads * max_splits), ctx.empty(m * heads * max_splits)
    pa = ctx.empty(m * heads * max_splits * d)
    out = ctx.empty((m, heads * d))

    # The oracle: each row's blocks as a ring, the stores, the ring attention.
    kr, vr = MC.pool_to_rings(kpool, tables), MC.pool_to_rings(vpool, tables)
    length, rows = table_len * block_size, np.arange(m, dtype=np.uint32)
    krot = O.rope(qkv[:, heads * d:(heads + kv_heads) * d], kv_heads, d, d // 2, pos, cos_t, sin_t)
    O.kv_store_ring(MC.rounded(t, krot), kv_heads, d, length, pos, rows, kr)
    O.kv_store_ring(MC.rounded(t, np.ascontiguousarray(qkv[:, (heads + kv_heads) * d:])), kv_heads, d, length, pos,
                    rows, vr)
    kwant, vwant = kpool.copy(), vpool.copy()
    MC.rings_to_pool(kr, tables, kwant)
    MC.rings_to_pool(vr, tables, vwant)
    qrot = O.rope(qkv[:, :heads * d], heads, d, d // 2, pos, cos_t, sin_t)
    want, _ = O.attend(qrot, heads, kv_heads, d, length, pos, rows, kr, vr, np.float32(1.0 / math.sqrt(d)), chunk,
                       4, max_splits, THREADS)

    def stored_as_wanted(kb, vb):
        kgot, vgot = gathered(kb, shape, dtype), gathered(vb, shape, dtype)
        if t != "f32":
            return (np.array_equal(kgot, MC.narrow(t, kwant).reshape(shape))
                    and np.array_equal(vgot, MC.narrow(t, vwant).reshape(shape)))
        return same_bits(kgot, kwant) and same_bits(vgot, vwant)

    for fused in (False, True):
        kb, kkeep = scattered_blocks(ctx, kbits, 135 + fused)
        vb, vkeep = scattered_blocks(ctx, vbits, 136 + fused)
        dkt = ctx.to_device(np.array([b.ptr for b in kb], np.uint64))
        dvt = ctx.to_device(np.array([b.ptr for b in vb], np.uint64))
        attend = dict(pg, m=m, heads=heads, kv_heads=kv_heads, d=d, rotated=d // 2, chunk=chunk,
                      max_splits=max_splits, ldq=width, q_off=0, scale=1.0 / math.sqrt(d))
        if fused:
            ctx.launch("attend_decode_paged" + suffix, dict(attend, k_off=heads * d, v_off=(heads + kv_heads) * d),
                       [dq, dcos, dsin, dpos, dtab, pm, pl, pa, dkt, dvt])
        else:
            ctx.launch("kv_store_paged" + suffix,
                       dict(pg, m=m, kv_heads=kv_heads, d=d, rotated=d // 2, ldq=width, k_off=heads * d,
                            v_off=(heads + kv_heads) * d), [dq, dcos, dsin, dpos, dtab, dkt, dvt])
            ctx.launch("attend_split_paged" + suffix, attend, [dq, dcos, dsin, dpos, dtab, pm, pl, pa, dkt, dvt])
        ctx.launch("attend_combine", {"m": m, "heads": heads, "d": d, "chunk": chunk, "max_splits": max_splits,
                                      "ldo": heads * d}, [pm, pl, pa, dpos, out])
        assert same_bits(out.download(), want), fused
        assert stored_as_wanted(kb, vb), fused
        for b in kkeep + vkeep + [dkt, dvt]:
            b.free()
    for b in (dq, dpos, dtab, dcos, dsin, pm, pl, pa, out):
        b.free()


def test_paged_model_decode_step_blocks_allocated_apart(ctx):
    """A model's paged caches moved into blocks allocated one by one, out of
    order, and the engine's block-address tables pointed at them
    (set_block_addresses), the pool zeroed: the captured decode step gives
    the oracle's ids, logits and rows bit for bit, and the blocks hold the
    oracle's stores."""
    from furykernel_b200 import _native as N
    from furykernel_b200.engine import Llama
    from furykernel_b200.shape import LlamaShape

    batch = 2
    s = LlamaShape(d_model=512, heads=4, kv_heads=4, head_dim=128, ffn=1024, vocab=3000, layers=2, positions=96,
                   blocks=6 * batch + 3, block_size=16)
    eng = Llama(ctx, s, batch, seed=431, chunk=32, prefill_kv=1.0)
    tokens = O.ints(432, batch, s.vocab)
    pos = np.array([17, 90], np.uint32)
    tables = disjoint_tables(433, batch, s.table_len, s.blocks)
    layers, embed, final_norm = MC.host_model(eng)
    kc, vc = MC.host_caches(eng)  # [layers, blocks, kv_heads, bs, d]
    keep, moved = [], []
    for l in range(s.layers):
        kb, kk = scattered_blocks(ctx, kc[l], 440 + l)
        vb, vk = scattered_blocks(ctx, vc[l], 450 + l)
        eng.set_block_addresses(l, [b.ptr for b in kb], [b.ptr for b in vb])
        keep += kk + vk
        moved.append((kb, vb))
    n = s.layers * s.blocks * s.kv_heads * s.block_size * s.head_dim
    N.check(N.lib().fkc_buf_zero(ctx.handle, eng.kbase, 4 * n))  # the pool no longer holds the caches
    N.check(N.lib().fkc_buf_zero(ctx.handle, eng.vbase, 4 * n))
    eng.set_rows(tokens, pos, tables)
    ids = eng.step()
    want_ids, want_logits, want_x = MC.oracle_decode(eng, layers, embed, final_norm, kc, vc, tokens, pos, tables)
    assert np.array_equal(ids, want_ids)
    assert same_bits(eng.logits.download(), want_logits)
    assert same_bits(eng.x.download(), want_x)
    shape = kc.shape[1:]
    for l, (kb, vb) in enumerate(moved):
        assert same_bits(gathered(kb, shape, np.float32), kc[l]) and same_bits(gathered(vb, shape, np.float32), vc[l])
    for b in keep:
        b.free()
