"""Test infrastructure: a decode step of the Llama-shaped model recomputed by
the oracle -- bit for bit in the CPU target's arithmetic (fko_*), and in f64
with binary32 bounds (fkr_*, the reference's evaluator) -- from the weights
and caches the device holds."""

from __future__ import annotations

import math

import numpy as np

from oracle import oracle as O


def widen(t: str, bits) -> np.ndarray:
    """16-bit elements of type t ("bf16", "f16") as f32, exactly."""
    return O.widen_bf16(bits) if t == "bf16" else O.widen_f16(bits)


def narrow(t: str, a) -> np.ndarray:
    """f32 values rounded to type t ("bf16", "f16"), as its bits."""
    return O.narrow_bf16(a) if t == "bf16" else O.narrow_f16(a)


def rounded(t: str, a) -> np.ndarray:
    """f32 values as an element of type t holds them."""
    a = np.asarray(a, np.float32)
    return a if t == "f32" else widen(t, narrow(t, a)).reshape(a.shape)


def download_f32(eng, ptr, n, t):
    """n elements of type t ("f32", "bf16", "f16") at a device address as
    f32: 16-bit ones widened (exact)."""
    from furykernel_b200 import _native as N

    raw = np.empty(n, np.float32 if t == "f32" else np.uint16)
    N.check(N.lib().fkc_buf_download(eng.ctx.handle, raw.ctypes.data, ptr, raw.nbytes))
    return raw if t == "f32" else widen(t, raw)


def host_model(eng):
    """The engine's weights, per layer, as the device holds them (16-bit
    weights widened to f32, exactly)."""
    s = eng.s
    d, qw, kvw, f = s.d_model, s.q_width, s.kv_width, s.ffn
    wb = getattr(eng, "wb", 4)
    flat = download_f32(eng, eng.arena.ptr, eng.arena.nbytes // wb, s.weights)
    layers = []
    for l in range(s.layers):
        base = l * eng.layer_elems
        at = base
        w = {}
        e = getattr(s, "experts", 0)
        scale = [("expert_scale", 1, e)] if e and getattr(s, "expert_scale", False) else []
        ffn = [("router", e, d)] + scale + [("egu", e * 2 * f, d), ("edn", e * d, f)] if e else \
            [("gu", 2 * f, d), ("down", d, f)]
        for name, rows, cols in [("qkv", qw + 2 * kvw, d), ("o", d, qw)] + ffn + [("attn_norm", 1, d),
                                                                                   ("mlp_norm", 1, d)]:
            w[name] = flat[at:at + rows * cols].reshape(rows, cols) if rows > 1 else flat[at:at + cols].copy()
            at += rows * cols
        if e:  # the experts' tables, an entry each
            w["egu"] = w["egu"].reshape(e, 2 * f, d)
            w["edn"] = w["edn"].reshape(e, d, f)
        elif eng.gate_up_interleaved:  # rows gate_0, up_0, gate_1, ...: back to [gate; up]
            w["gu"] = np.ascontiguousarray(np.concatenate([w["gu"][0::2], w["gu"][1::2]]))
        layers.append(w)
    e0 = s.layers * eng.layer_elems
    embed = flat[e0:e0 + s.vocab * d].reshape(s.vocab, d)
    final_norm = flat[e0 + s.vocab * d:e0 + s.vocab * d + d].copy()
    return layers, embed, final_norm


def host_caches(eng):
    """The KV caches as the device holds them, as f32 (16-bit widened):
    [layers, slots, kv_heads, length, d] rings, or [layers, blocks,
    kv_heads, block_size, d] pools."""
    s = eng.s
    units, unit_len = (s.blocks, s.block_size) if getattr(s, "paged", False) else (s.slots, s.length)
    n = s.layers * units * s.kv_heads * unit_len * s.head_dim
    k = download_f32(eng, eng.kbase, n, s.cache)
    v = download_f32(eng, eng.vbase, n, s.cache)
    shp = (s.layers, units, s.kv_heads, unit_len, s.head_dim)
    return k.reshape(shp), v.reshape(shp)


def pool_to_rings(pool, tables):
    """A layer's paged pool [blocks, kv_heads, bs, d] as one ring a row
    [m, kv_heads, table_len * bs, d]: row r's blocks in its table's order,
    so that position t of the row is ring position t (cacheIndex,
    src/FuryKernel/Program/Eval.hs:592-602)."""
    tables = np.asarray(tables)
    m, tl = tables.shape
    _, kvh, bs, d = pool.shape
    g = pool[tables.reshape(-1)].reshape(m, tl, kvh, bs, d)
    return np.ascontiguousarray(g.transpose(0, 2, 1, 3, 4).reshape(m, kvh, tl * bs, d))


def rings_to_pool(rings, tables, pool):
    """The rows' rings written back into the pool through their tables."""
    tables = np.asarray(tables)
    m, tl = tables.shape
    _, kvh, bs, d = pool.shape
    blocks = rings.reshape(m, kvh, tl, bs, d).transpose(0, 2, 1, 3, 4).reshape(m * tl, kvh, bs, d)
    pool[tables.reshape(-1)] = blocks


def splits_of(eng):
    """The split-K of each GEMV launch, in launch order."""
    return [L.params["split"] for L in eng.launches if L.kernel.startswith("gemv")]


def oracle_decode(eng, layers, embed, final_norm, kcache, vcache, tokens, pos, slot, threads=0):
    """The CPU target's bits for one decode step; the caches are updated in
    place as the step's stores leave them (16-bit caches: each stored element
    rounded to the cache's type, Eval.hs:9). Returns (ids, logits, x)."""
    s = eng.s

    def as_stored(a):
        return rounded(s.cache, a)

    threads = threads or O.threads_default()
    d, qw, kvw, f, hd = s.d_model, s.q_width, s.kv_width, s.ffn, s.head_dim
    cos_t, sin_t = O.rope_tables(s.theta, hd, hd // 2, s.positions)
    splits = iter(splits_of(eng))
    scale = np.float32(1.0 / math.sqrt(hd))
    eps = np.float32(s.eps)
    x = O.gather(embed, tokens)
    for l, w in enumerate(layers):
        a = O.rmsnorm_rows(x, w["attn_norm"], eps, 1.0, threads)
        qkv = O.gemv(w["qkv"], a, next(splits), threads)
        q, k, v = qkv[:, :qw], qkv[:, qw:qw + kvw], qkv[:, qw + kvw:]
        kr = O.rope(k, s.kv_heads, hd, hd // 2, pos, cos_t, sin_t)
        if getattr(s, "paged", False):  # `slot` holds the rows' block tables
            kc, vc = pool_to_rings(kcache[l], slot), pool_to_rings(vcache[l], slot)
            length, rslot = s.table_len * s.block_size, np.arange(len(pos), dtype=np.uint32)
        else:
            kc, vc, length, rslot = kcache[l], vcache[l], s.length, slot
        O.kv_store_ring(as_stored(kr), s.kv_heads, hd, length, pos, rslot, kc)
        O.kv_store_ring(as_stored(np.ascontiguousarray(v)), s.kv_heads, hd, length, pos, rslot, vc)
        if getattr(s, "paged", False):
            rings_to_pool(kc, slot, kcache[l])
            rings_to_pool(vc, slot, vcache[l])
        qr = O.rope(q, s.heads, hd, hd // 2, pos, cos_t, sin_t)
        att, _ = O.attend(qr, s.heads, s.kv_heads, hd, length, pos, rslot, kc, vc, scale, eng.chunk, 4,
                          eng.max_splits, threads)
        x1 = O.add(x, O.gemv(w["o"], att, next(splits), threads))
        if getattr(s, "experts", 0):  # the router, the top k, the experts' GELU-gated FFNs, their weighted sum
            m_in = O.rmsnorm_rows(x1, w["mlp_norm"], eps, 1.0, threads)
            logits = O.gemv(w["router"], m_in, next(splits), threads)
            ids, ws = O.route_topk(logits, s.top_k, w.get("expert_scale"))
            gu = O.gemv_routed(w["egu"], ids, m_in, next(splits), threads)
            eo = O.gemv_routed(w["edn"], ids, O.gated_gelu(gu, f), next(splits), threads)
            x = O.combine_ranks_add(x1, ws, eo)
            continue
        gu = O.gemv(w["gu"], O.rmsnorm_rows(x1, w["mlp_norm"], eps, 1.0, threads), next(splits), threads)
        act = O.silu_mul(gu[:, :f], gu[:, f:])
        x = O.add(x1, O.gemv(w["down"], act, next(splits), threads))
    logits = O.gemv(embed, O.rmsnorm_rows(x, final_norm, eps, 1.0, threads), next(splits), threads)
    return O.argmax(logits), logits, x


def oracle_decode_tp(s, world, layers, embed, final_norm, kcache, vcache, tokens, pos, slot, chunk, max_splits,
                     threads=0):
    """The CPU target's bits for one tensor-parallel decode step over the
    peer exchange: each rank's shard GEMVs in the contract's order over its
    own slice, the row-parallel partials added in rank order, then the
    residual: x1 = x + (((P_0 + P_1) + ...)). `layers` holds the whole
    model (q, k, v, o, gate, up, down, attn_norm, mlp_norm per layer; with
    routed experts router, egu and edn in place of gate, up and down: every
    rank routes with the whole router, runs its ffn slice of each chosen
    expert, and the ranks' expert outputs are added in rank order before
    the combine); the caches [layers, slots, kv_heads, length, hd] are
    updated in place. Returns (ids, logits, x)."""
    threads = threads or O.threads_default()
    d, hd = s.d_model, s.head_dim
    hq, hk, fl, vl = s.heads // world, s.kv_heads // world, s.ffn // world, s.vocab // world
    cos_t, sin_t = O.rope_tables(s.theta, hd, hd // 2, s.positions)
    scale = np.float32(1.0 / math.sqrt(hd))
    eps = np.float32(s.eps)
    x = O.gather(embed, tokens)

    def ranked_sum(parts):
        total = parts[0]
        for p in parts[1:]:
            total = O.add(total, p)
        return total

    for l, w in enumerate(layers):
        a = O.rmsnorm_rows(x, w["attn_norm"], eps, 1.0, threads)
        parts = []
        for r in range(world):
            qs, ks = slice(r * hq * hd, (r + 1) * hq * hd), slice(r * hk * hd, (r + 1) * hk * hd)
            wqkv = np.concatenate([w["q"][qs], w["k"][ks], w["v"][ks]])
            qkv = O.gemv(wqkv, a, 1, threads)
            q, k, v = qkv[:, :hq * hd], qkv[:, hq * hd:(hq + hk) * hd], qkv[:, (hq + hk) * hd:]
            kc = np.ascontiguousarray(kcache[l][:, r * hk:(r + 1) * hk])
            vc = np.ascontiguousarray(vcache[l][:, r * hk:(r + 1) * hk])
            O.kv_store_ring(O.rope(k, hk, hd, hd // 2, pos, cos_t, sin_t), hk, hd, s.length, pos, slot, kc)
            O.kv_store_ring(np.ascontiguousarray(v), hk, hd, s.length, pos, slot, vc)
            kcache[l][:, r * hk:(r + 1) * hk] = kc
            vcache[l][:, r * hk:(r + 1) * hk] = vc
            qr = O.rope(q, hq, hd, hd // 2, pos, cos_t, sin_t)
            att, _ = O.attend(qr, hq, hk, hd, s.length, pos, slot, kc, vc, scale, chunk, 4, max_splits, threads)
            parts.append(O.gemv(np.ascontiguousarray(w["o"][:, qs]), att, 1, threads))
        x1 = O.add(x, ranked_sum(parts))
        m2 = O.rmsnorm_rows(x1, w["mlp_norm"], eps, 1.0, threads)
        parts = []
        if getattr(s, "experts", 0):
            ids, ws = O.route_topk(O.gemv(w["router"], m2, 1, threads), s.top_k, w.get("expert_scale"))
            for r in range(world):
                egu = np.ascontiguousarray(np.concatenate(
                    [w["egu"][:, r * fl:(r + 1) * fl], w["egu"][:, s.ffn + r * fl:s.ffn + (r + 1) * fl]], axis=1))
                edn = np.ascontiguousarray(w["edn"][:, :, r * fl:(r + 1) * fl])
                gu = O.gemv_routed(egu, ids, m2, 1, threads)
                parts.append(O.gemv_routed(edn, ids, O.gated_gelu(gu, fl), 1, threads))
            x = O.combine_ranks_add(x1, ws, ranked_sum(parts))
            continue
        for r in range(world):
            fs = slice(r * fl, (r + 1) * fl)
            g = O.gemv(w["gate"][fs], m2, 1, threads)
            u = O.gemv(w["up"][fs], m2, 1, threads)
            parts.append(O.gemv(np.ascontiguousarray(w["down"][:, fs]), O.silu_mul(g, u), 1, threads))
        x = O.add(x1, ranked_sum(parts))
    n = O.rmsnorm_rows(x, final_norm, eps, 1.0, threads)
    logits = np.concatenate([O.gemv(embed[r * vl:(r + 1) * vl], n, 1, threads) for r in range(world)], axis=1)
    return O.argmax(logits), logits, x


def may_store(t, exact, bound, got) -> bool:
    """Whether a kernel may have stored `got` for elements of the given
    exact values and bounds in a cache of type t (mayStore,
    src/FuryKernel/Program/Eval.hs:924-944): an unbounded element anything;
    a NaN exact value a NaN; else, f32: within the widened bound; 16-bit:
    between the roundings to t of the exact value less and plus it."""
    exact, bound, got = (np.asarray(a, np.float64) for a in (exact, bound, got))
    e = O.widened(bound)
    free = np.isinf(bound)
    nan = np.isnan(exact) & ~free
    rest = ~free & ~nan
    if t == "f32":
        ok = np.abs(got[rest] - exact[rest]) <= e[rest]
    else:
        lo, hi = O.round_to(t, exact[rest] - e[rest]), O.round_to(t, exact[rest] + e[rest])
        ok = (lo <= got[rest]) & (got[rest] <= hi)
    return bool(np.all(ok) and np.all(np.isnan(got[nan])))


def referee_decode(eng, layers, embed, final_norm, kcache_after, vcache_after, tokens, pos, slot):
    """The f64 evaluator's values and bounds for the same step, attention
    reading the caches as the kernels left them (evaluateStored,
    Eval.hs:186-198). Returns ((logits, bounds), (ids, decided), kv checks)."""
    s = eng.s
    d, qw, kvw, f, hd = s.d_model, s.q_width, s.kv_width, s.ffn, s.head_dim
    x = O.r_gather(embed, tokens)
    stored_ok = True
    for l, w in enumerate(layers):
        a = O.r_rmsnorm(x, d, w["attn_norm"], s.eps)
        qkv = O.r_linear(w["qkv"], a)
        q = (qkv[0][:, :qw], qkv[1][:, :qw])
        k = (qkv[0][:, qw:qw + kvw], qkv[1][:, qw:qw + kvw])
        v = (qkv[0][:, qw + kvw:], qkv[1][:, qw + kvw:])
        kr = O.r_rope(k, hd, hd // 2, s.theta, pos)
        kc, vc = kcache_after[l], vcache_after[l]
        for r in range(len(pos)):  # the stores the kernels made lie within their bounds
            for h in range(s.kv_heads):
                at = (slot[r], h, pos[r] % s.length)
                for vals, cache in ((kr, kc), (v, vc)):
                    exact = vals[0][r, h * hd:(h + 1) * hd]
                    bound = vals[1][r, h * hd:(h + 1) * hd]
                    got = cache[at].astype(np.float64)
                    stored_ok &= may_store(s.cache, exact, bound, got)
        qr = O.r_rope(q, hd, hd // 2, s.theta, pos)
        att = O.r_attend(qr, s.heads, s.kv_heads, hd, s.length, pos, slot, kc.astype(np.float64),
                         vc.astype(np.float64), 1.0 / math.sqrt(hd))
        x1 = O.r_add(x, O.r_linear(w["o"], att))
        gu = O.r_linear(w["gu"], O.r_rmsnorm(x1, d, w["mlp_norm"], s.eps))
        act = O.r_silu_mul((gu[0][:, :f], gu[1][:, :f]), (gu[0][:, f:], gu[1][:, f:]))
        x = O.r_add(x1, O.r_linear(w["down"], act))
    logits = O.r_linear(embed, O.r_rmsnorm(x, d, final_norm, s.eps))
    return logits, O.r_argmax(logits), stored_ok
