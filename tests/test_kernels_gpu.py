"""Parity of each CUDA kernel with the oracle, through the C ABI, on a B200.

The CUDA kernels keep the spec kernels' arithmetic order, so most outputs
are compared bit for bit with the oracle's restatement of the reference CPU
target (oracle/fko_cpu.c). Every f32 output is also checked against the f64
evaluator's per-element bound (oracle/fko_eval.c, Eval.hs), and, per the
path's tolerances, by its normwise relative error against the f64 value:
max |gpu - exact| / max |exact| <= 1e-5 for elementwise and norm kernels,
<= 1e-4 for reductions, GEMV and attention.
"""

import math

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

THREADS = O.threads_default()


@pytest.fixture(scope="module")
def ctx():
    from furykernel_b200 import _native as N

    c = N.Context(0)
    yield c
    c.close()


def rel_err(got, exact):
    got = np.asarray(got, np.float64)
    return float(np.max(np.abs(got - exact)) / max(np.max(np.abs(exact)), 1e-300))


def same_bits(a, b):
    a = np.ascontiguousarray(a, np.float32).view(np.uint32)
    b = np.ascontiguousarray(b, np.float32).view(np.uint32)
    return a.shape == b.shape and np.array_equal(a, b)


# ---------------------------------------------------------------------------
# Config 1: the threadgroup tree reduction


def run_reduce(ctx, x):
    xd = ctx.to_device(x)
    groups = (x.size + 255) // 256
    part = ctx.empty(groups)
    y = ctx.empty(1)
    ctx.launch("reduce_groups", {"n": x.size}, [xd, part])
    ctx.launch("reduce_final", {"count": groups}, [part, y])
    out = y.download()[0], part.download()
    for b in (xd, part, y):
        b.free()
    return out


@pytest.mark.parametrize("n", [1, 255, 256, 65536, 65536 + 17, 16_777_216])
def test_reduce_bit_exact(ctx, n):
    x = O.uniform(2026 + n, n, -1.0, 1.0)
    got, part = run_reduce(ctx, x)
    assert same_bits(part, O.reduce_partials(x, THREADS))
    want = O.reduce_sum(x, THREADS)
    assert same_bits([got], [want]), (got, want)
    exact, bound = O.r_sum(x)
    assert abs(float(got) - exact) <= O.widened(bound)


def test_reduce_of_negative_zeros_is_negative_zero(ctx):
    got, _ = run_reduce(ctx, np.full(1000, -0.0, np.float32))
    assert np.float32(got).view(np.uint32) == 0x80000000


def test_reduce_known_order(ctx):
    # 2^24 at element 0 and ones at 16 and 17 of a group: the halving tree
    # meets the two ones first only where the tree says (spec of config 1).
    x = np.zeros(256, np.float32)
    x[0] = 2.0 ** 24
    x[1] = x[129] = 1.0  # halving by 128 adds them first: 2 + 2^24 survives
    got, _ = run_reduce(ctx, x)
    assert got == O.reduce_sum(x) == np.float32(2.0 ** 24 + 2)


# ---------------------------------------------------------------------------
# Config 2: RMSNorm then softmax over rows


@pytest.mark.parametrize("rows,h", [(3, 1000), (64, 4096), (4096, 4096)])
def test_rmsnorm_softmax_rows(ctx, rows, h):
    x = O.normal(11, rows * h).reshape(rows, h)
    gamma = O.uniform(12, h, 0.5, 1.5)
    xd, gd = ctx.to_device(x), ctx.to_device(gamma)
    yd, zd = ctx.empty((rows, h)), ctx.empty((rows, h))
    ctx.launch("rmsnorm_rows", {"rows": rows, "h": h, "eps": 1e-5, "factor": 1.0}, [xd, gd, yd])
    ctx.launch("softmax_rows", {"rows": rows, "h": h}, [yd, zd])
    y, z = yd.download(), zd.download()
    y_cpu = O.rmsnorm_rows(x, gamma, 1e-5, 1.0, THREADS)
    assert same_bits(y, y_cpu)
    z_cpu = O.softmax_rows(y_cpu, THREADS)
    # exp is binary64's on both sides, rounded once: CUDA's and glibc's
    # binary64 exp may round an element differently; none did on the seeds here.
    assert same_bits(z, z_cpu)
    if rows <= 64:
        ref = O.r_rmsnorm(O.r_input(x), h, gamma, 1e-5)
        assert O.within(y, ref).all()
        assert rel_err(y, ref[0]) <= 1e-5
        sref = O.r_softmax(O.r_input(y))
        assert O.within(z, sref).all()
        assert rel_err(z, sref[0]) <= 1e-5
    for b in (xd, gd, yd, zd):
        b.free()


# ---------------------------------------------------------------------------
# Config 3a/3b: GEMV, and the plan's prologue and epilogue variants


@pytest.mark.parametrize("n,k,m,split", [(11008, 4096, 1, 1), (11008, 4096, 16, 1), (4096, 11008, 1, 2),
                                         (300, 1000, 3, 4), (257, 4096, 32, 8), (11008, 4096, 5, 1),
                                         (4096, 11008, 32, 1), (1001, 1000, 64, 1), (22, 4100, 9, 1),
                                         (3, 256, 17, 1)])
def test_gemv_bit_exact(ctx, n, k, m, split):
    w = O.normal(21, n * k, 0.0, 0.02).reshape(n, k)
    x = O.normal(22, m * k).reshape(m, k)
    wd, xd, yd = ctx.to_device(w), ctx.to_device(x), ctx.empty((m, n))
    ctx.launch("gemv", {"n": n, "k": k, "m": m, "split": split, "ldx": k, "ldy": n}, [wd, xd, yd])
    y = yd.download()
    assert same_bits(y, O.gemv(w, x, split, THREADS))
    if n * k * m <= 11008 * 4096:
        ref = O.r_linear(w, O.r_input(x))
        assert O.within(y, ref).all()
        assert rel_err(y, ref[0]) <= 1e-4
    for b in (wd, xd, yd):
        b.free()


def test_gemv_prologues_and_epilogue(ctx):
    n, k, m = 1000, 2048, 4
    w = O.normal(31, n * k, 0.0, 0.02).reshape(n, k)
    x = O.normal(32, m * k).reshape(m, k)
    g = O.uniform(33, k, 0.5, 1.5)
    r = O.normal(34, m * n).reshape(m, n)
    gu = O.normal(35, m * 2 * k).reshape(m, 2 * k)
    wd, xd, gd, rd, gud = (ctx.to_device(a) for a in (w, x, g, r, gu))
    yd = ctx.empty((m, n))
    base = {"n": n, "k": k, "m": m, "split": 2, "ldx": k, "ldy": n}
    # RMSNorm recomputed before the anchor.
    ctx.launch("gemv_rmsnorm", dict(base, eps=1e-5, factor=1.0), [wd, xd, gd, yd])
    want = O.gemv(w, O.rmsnorm_rows(x, g, 1e-5), 2, THREADS)
    assert same_bits(yd.download(), want)
    # The residual added on the tile.
    ctx.launch("gemv_add", dict(base, ldr=n), [wd, xd, rd, yd])
    assert same_bits(yd.download(), O.add(r, O.gemv(w, x, 2, THREADS)))
    # SiLU-gate recomputed from a stored gate/up row, then the residual.
    ctx.launch("gemv_silu_add", dict(base, ldx=2 * k, ldr=n, up_off=k), [wd, gud, rd, yd])
    act = O.silu_mul(gu[:, :k], gu[:, k:])
    assert same_bits(yd.download(), O.add(r, O.gemv(w, act, 2, THREADS)))
    ctx.launch("gemv_silu", dict(base, ldx=2 * k, up_off=k), [wd, gud, yd])
    assert same_bits(yd.download(), O.gemv(w, act, 2, THREADS))
    for b in (wd, xd, gd, rd, gud, yd):
        b.free()


@pytest.mark.parametrize("m", [6, 12, 40])
def test_batched_gemv_prologue_and_epilogues(ctx, m):
    """The batched kernel (5 to 64 rows, split 1): RMSNorm before the
    anchor, the residual on the tile, and the SiLU-gate of interleaved
    gate/up rows on the pair's tile."""
    n, k = 1002, 2048
    w = O.normal(41, n * k, 0.0, 0.02).reshape(n, k)
    x = O.normal(42, m * k).reshape(m, k)
    g = O.uniform(43, k, 0.5, 1.5)
    r = O.normal(44, m * n).reshape(m, n)
    wd, xd, gd, rd = (ctx.to_device(a) for a in (w, x, g, r))
    yd = ctx.empty((m, n))
    base = {"n": n, "k": k, "m": m, "split": 1, "ldx": k, "ldy": n}
    ctx.launch("gemv_rmsnorm", dict(base, eps=1e-5, factor=1.0), [wd, xd, gd, yd])
    normed = O.rmsnorm_rows(x, g, 1e-5)
    assert same_bits(yd.download(), O.gemv(w, normed, 1, THREADS))
    ctx.launch("gemv_add", dict(base, ldr=n), [wd, xd, rd, yd])
    assert same_bits(yd.download(), O.add(r, O.gemv(w, x, 1, THREADS)))
    ad = ctx.empty((m, n // 2))
    ctx.launch("gemv_rmsnorm_silu", dict(base, ldy=n // 2, eps=1e-5, factor=1.0), [wd, xd, gd, ad])
    want = O.silu_mul(O.gemv(np.ascontiguousarray(w[0::2]), normed, 1, THREADS),
                      O.gemv(np.ascontiguousarray(w[1::2]), normed, 1, THREADS))
    assert same_bits(ad.download(), want)
    for b in (wd, xd, gd, rd, yd, ad):
        b.free()


def test_batched_gemv_subnormal_and_special_values(ctx):
    """The packed f32x2 arithmetic keeps subnormal products and sums (no
    flush to zero) and carries infinities and NaNs as the scalar one does."""
    n, k, m = 64, 512, 10
    w = O.normal(51, n * k, 0.0, 0.02).reshape(n, k)
    x = O.normal(52, m * k).reshape(m, k)
    x[1] *= np.float32(1e-38)   # products and sums in the subnormal range
    x[2] *= np.float32(1e-30)
    x[3, 7] = np.float32(np.inf)
    x[4, 9] = np.float32(np.nan)
    x[5, 11] = np.float32(-np.inf)
    x[5, 12] = np.float32(np.inf)
    wd, xd, yd = ctx.to_device(w), ctx.to_device(x), ctx.empty((m, n))
    ctx.launch("gemv", {"n": n, "k": k, "m": m, "split": 1, "ldx": k, "ldy": n}, [wd, xd, yd])
    y = yd.download()
    want = O.gemv(w, x, 1, THREADS)
    assert np.any((y[1] != 0) & (np.abs(y[1]) < np.finfo(np.float32).tiny))
    # NaN payloads aside, the same values bit for bit.
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(y), nan)
    assert same_bits(np.where(nan, 0, y), np.where(nan, 0, want))
    for b in (wd, xd, yd):
        b.free()


@pytest.mark.parametrize("n,k,m,pack,split", [(11008, 4096, 1, 8, 1), (4096, 11008, 4, 8, 2), (300, 1024, 3, 4, 4),
                                              (257, 2048, 16, 16, 1), (64, 512, 7, 16, 8), (33, 96, 2, 4, 16)])
def test_gemv_bf16_family_bit_exact(ctx, n, k, m, pack, split):
    """The reference's bf16 GEMV family (Gemv.hs): bf16 in and out, f32
    chains, the oracle's bits for every pack width and split."""
    w = O.narrow_bf16(O.normal(81, n * k, 0.0, 0.02)).reshape(n, k)
    x = O.narrow_bf16(O.normal(82, m * k)).reshape(m, k)
    wd, xd = ctx.to_device(w), ctx.to_device(x)
    yd = ctx.empty((m, n), np.uint16)
    ctx.launch("gemv_bf16", {"n": n, "k": k, "m": m, "pack": pack, "split": split, "ldx": k, "ldy": n}, [wd, xd, yd])
    assert np.array_equal(yd.download(), O.gemv_bf16(w, x, pack, split, THREADS))
    for b in (wd, xd, yd):
        b.free()


def test_gemv_bf16_special_values(ctx):
    n, k, m = 40, 256, 3
    w = O.narrow_bf16(O.normal(83, n * k, 0.0, 0.02)).reshape(n, k)
    x = O.narrow_bf16(O.normal(84, m * k)).reshape(m, k)
    x[0, 5] = 0x7F80  # +inf
    x[1, 9] = 0x7FC1  # a NaN
    x[2] = O.narrow_bf16(O.widen_bf16(x[2]) * np.float32(1e-38))  # subnormal products
    wd, xd = ctx.to_device(w), ctx.to_device(x)
    yd = ctx.empty((m, n), np.uint16)
    ctx.launch("gemv_bf16", {"n": n, "k": k, "m": m, "pack": 8, "split": 1, "ldx": k, "ldy": n}, [wd, xd, yd])
    got, want = yd.download(), O.gemv_bf16(w, x, 8, 1)
    nan = np.isnan(O.widen_bf16(want))
    assert np.array_equal(np.isnan(O.widen_bf16(got)), nan)  # NaN payloads aside
    assert np.array_equal(got[~nan], want[~nan])
    for b in (wd, xd, yd):
        b.free()


# ---------------------------------------------------------------------------
# The decode attention path: KV store, split attention, combine


@pytest.mark.parametrize("m,heads,kv_heads,length,positions,chunk", [
    (2, 4, 2, 64, [5, 40], 16),
    (3, 8, 8, 300, [0, 129, 299], 64),
    (1, 32, 32, 2304, [2048], 128),
    (4, 4, 4, 40, [45, 3, 39, 80], 32),  # positions past the ring's length wrap
    # The combine holds 32 splits in registers, then loads 8 at a time, then one:
    # 32 and 34 splits at the boundary, 66 through all three.
    (2, 4, 4, 1100, [1023, 1056], 32),
    (1, 4, 2, 2304, [2100], 32),
    # The KV store takes 4 heads a block: 6 leave the second block half idle.
    (2, 12, 6, 64, [10, 50], 16),
])
def test_attention_path(ctx, m, heads, kv_heads, length, positions, chunk):
    d = 128
    slots = m
    width = (heads + 2 * kv_heads) * d
    qkv = O.normal(41, m * width).reshape(m, width)
    pos = np.array(positions, np.uint32)
    slot = np.arange(m, dtype=np.uint32)[::-1].copy()
    kc = O.normal(42, slots * kv_heads * length * d).reshape(slots, kv_heads, length, d)
    vc = O.normal(43, slots * kv_heads * length * d).reshape(slots, kv_heads, length, d)
    maxpos = int(pos.max()) + 1
    cos_t, sin_t = O.rope_tables(10000.0, d, d // 2, maxpos)
    max_splits = (maxpos + chunk - 1) // chunk

    dq, dkc, dvc, dpos, dslot = (ctx.to_device(a) for a in (qkv, kc, vc, pos, slot))
    dcos, dsin = ctx.rope_tables(10000.0, d, d // 2, maxpos)
    assert same_bits(dcos.download(), cos_t) and same_bits(dsin.download(), sin_t)
    pm = ctx.empty(m * heads * max_splits)
    pl = ctx.empty(m * heads * max_splits)
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

    # The oracle: rope(k) and v stored, then split attention and combine.
    kcache, vcache = kc.copy(), vc.copy()
    krot = O.rope(qkv[:, heads * d:(heads + kv_heads) * d], kv_heads, d, d // 2, pos, cos_t, sin_t)
    O.kv_store_ring(krot, kv_heads, d, length, pos, slot, kcache)
    O.kv_store_ring(np.ascontiguousarray(qkv[:, (heads + kv_heads) * d:]), kv_heads, d, length, pos, slot, vcache)
    assert same_bits(dkc.download(), kcache) and same_bits(dvc.download(), vcache)
    qrot = O.rope(qkv[:, :heads * d], heads, d, d // 2, pos, cos_t, sin_t)
    want, _ = O.attend(qrot, heads, kv_heads, d, length, pos, slot, kcache, vcache,
                       np.float32(1.0 / math.sqrt(d)), chunk, 4, max_splits, THREADS)
    got = out.download()
    assert same_bits(got, want)
    # The store and the attention as one launch (rows in distinct slots),
    # then the combine: the same bits, the same caches.
    dkc.upload(kc)
    dvc.upload(vc)
    out2 = ctx.empty((m, heads * d))
    ctx.launch("attend_decode", {"m": m, "heads": heads, "kv_heads": kv_heads, "d": d, "length": length,
                                 "rotated": d // 2, "chunk": chunk, "max_splits": max_splits, "ldq": width,
                                 "q_off": 0, "k_off": heads * d, "v_off": (heads + kv_heads) * d,
                                 "scale": 1.0 / math.sqrt(d)},
               [dq, dcos, dsin, dpos, dslot, dkc, dvc, pm, pl, pa])
    ctx.launch("attend_combine", {"m": m, "heads": heads, "d": d, "chunk": chunk, "max_splits": max_splits,
                                  "ldo": heads * d}, [pm, pl, pa, dpos, out2])
    assert same_bits(out2.download(), want)
    assert same_bits(dkc.download(), kcache) and same_bits(dvc.download(), vcache)
    out2.free()
    # The referee: attention over the caches as the kernels left them
    # (evaluateStored), positions <= pos; rows never wrap past `length` here
    # except the wrapping case, which reads the ring as stored.
    if all(p < length for p in positions):
        qref = O.r_rope(O.r_input(qkv[:, :heads * d]), d, d // 2, 10000.0, pos)
        ref = O.r_attend(qref, heads, kv_heads, d, length, pos, slot, kcache.astype(np.float64),
                         vcache.astype(np.float64), 1.0 / math.sqrt(d))
        assert O.within(got, ref).all()
        assert rel_err(got, ref[0]) <= 1e-4
    for b in (dq, dkc, dvc, dpos, dslot, dcos, dsin, pm, pl, pa, out):
        b.free()


# ---------------------------------------------------------------------------
# Elementwise, gather, argmax


def test_elementwise_and_gather(ctx):
    n = 100_000
    a, b = O.normal(51, n), O.normal(52, n)
    da, db, dy = ctx.to_device(a), ctx.to_device(b), ctx.empty(n)
    ctx.launch("add", {"n": n}, [da, db, dy])
    assert same_bits(dy.download(), O.add(a, b))
    # A count that is not a multiple of 4 takes the scalar form: the same sums.
    ctx.launch("add", {"n": n - 3}, [da, db, dy])
    assert same_bits(dy.download()[:n - 3], O.add(a[:n - 3], b[:n - 3]))
    ctx.launch("silu_mul", {"n": n}, [da, db, dy])
    assert same_bits(dy.download(), O.silu_mul(a, b))
    ref = O.r_silu_mul(O.r_input(a), O.r_input(b))
    assert O.within(dy.download(), ref).all()
    table = O.normal(53, 1000 * 64, 0.0, 0.02).reshape(1000, 64)
    toks = np.array([3, 999, 0, 3], np.uint32)
    dt, dtok, dg = ctx.to_device(table), ctx.to_device(toks), ctx.empty((4, 64))
    ctx.launch("gather", {"width": 64, "m": 4, "factor": 1.0}, [dt, dtok, dg])
    assert same_bits(dg.download(), O.gather(table, toks))
    for buf in (da, db, dy, dt, dtok, dg):
        buf.free()


# n, ldx: whole packs of 4 (the vectorised scan), a ragged tail after the
# packs, and rows that do not start on 16 bytes (the scalar scan).
@pytest.mark.parametrize("n,ldx", [(32000, 32000), (32002, 32004), (31999, 32003)])
def test_argmax_first_index_ties_and_nans(ctx, n, ldx):
    rows = []
    r = O.normal(61, n)
    rows.append(r.copy())
    t = r.copy()
    t[100] = t[31000] = 50.0  # a tie: the lower index
    rows.append(t)
    t = r.copy()
    t[0] = np.nan  # a NaN first: the fold keeps index 0
    rows.append(t)
    t = r.copy()
    t[5] = np.nan
    t[7] = 60.0  # NaNs later are never taken
    rows.append(t)
    t = np.full(n, -np.inf, np.float32)  # all equal: index 0
    rows.append(t)
    t = np.zeros(n, np.float32)
    t[3] = -0.0
    t[9] = 0.0  # +0 and -0 tie: the lower index
    rows.append(t)
    t = r.copy()
    t[n - 1] = 70.0  # the maximum in the last element (a ragged tail's, where there is one)
    rows.append(t)
    x = np.stack(rows)
    xp = np.zeros((len(rows), ldx), np.float32)
    xp[:, :n] = x
    dx, di = ctx.to_device(xp), ctx.empty(len(rows), np.uint32)
    ctx.launch("argmax", {"m": len(rows), "n": n, "ldx": ldx}, [dx, di])
    got = di.download()
    assert np.array_equal(got, O.argmax(x))
    assert list(got[1:]) == [100, 0, 7, 0, 0, n - 1]
    dx.free()
    di.free()


def test_rope_kernel(ctx):
    m, heads, d = 3, 5, 128
    x = O.normal(71, m * heads * d).reshape(m, heads * d)
    pos = np.array([0, 7, 4095], np.uint32)
    c, s = O.rope_tables(10000.0, d, 48, 4096)
    dx, dp, dc, ds, dy = ctx.to_device(x), ctx.to_device(pos), ctx.to_device(c), ctx.to_device(s), ctx.empty((m, heads * d))
    ctx.launch("rope", {"m": m, "heads": heads, "d": d, "rotated": 48, "ldx": heads * d, "ldy": heads * d},
               [dx, dp, dc, ds, dy])
    got = dy.download()
    assert same_bits(got, O.rope(x, heads, d, 48, pos, c, s))
    ref = O.r_rope(O.r_input(x), d, 48, 10000.0, pos)
    assert O.within(got, ref).all()
    for b in (dx, dp, dc, ds, dy):
        b.free()


# ---------------------------------------------------------------------------
# The boundary's refusals and graphs


def test_dimension_refusal_text(ctx):
    from furykernel_b200 import _native as N

    # Buffers large enough for the refused shapes, so that nothing could
    # reach past them even if a check were missing.
    x = ctx.empty(65536 * 8)
    y = ctx.empty(65536 * 8)
    with pytest.raises(N.Refused) as e:
        ctx.launch("softmax_rows", {"rows": 1, "h": 6}, [x, y])
    assert str(e.value) == "softmax_rows: the dimension h is 6, outside its range 4..16384 multiple of 4."
    with pytest.raises(N.Refused) as e:
        ctx.launch("gemv", {"n": 4, "k": 4, "m": 65536, "split": 1, "ldx": 4, "ldy": 4}, [x, x, y])
    assert str(e.value) == "gemv: the dimension m is 65536, outside its range 1..65535."
    with pytest.raises(N.Refused) as e:
        ctx.launch("gemv", {"n": 4, "k": 4, "m": 1, "split": 9, "ldx": 4, "ldy": 4}, [x, x, y])
    assert str(e.value) == "gemv: the dimension split is 9, outside its range 1..8."
    x.free()
    y.free()


def test_graph_capture_replays_launches(ctx):
    n = 1 << 16
    a, b = O.normal(81, n), O.normal(82, n)
    da, db, dy = ctx.to_device(a), ctx.to_device(b), ctx.empty(n)
    ctx.capture_begin()
    ctx.launch("add", {"n": n}, [da, db, dy])
    ctx.launch("add", {"n": n}, [dy, db, dy])
    g = ctx.capture_end()
    g.launch()
    ctx.sync()
    assert same_bits(dy.download(), O.add(O.add(a, b), b))
    ms = g.time(1, 3)
    assert ms > 0
    g.destroy()
    for buf in (da, db, dy):
        buf.free()


def test_peer_wait_runs_out_and_reports():
    """A tensor-parallel exchange whose other rank never writes: the wait
    gives up at the context's bound (here 100 us), the kernel returns, the
    status word says which exchange buffer (10 + buffer), and the context
    stays usable. Both "ranks'" regions are on this GPU; the second rank
    simply never runs, so its row count never comes."""
    import ctypes
    import time

    from furykernel_b200 import _native as N

    L = N.lib()
    c = N.Context(0)
    try:
        words = L.fkc_peer_region_bytes() // 4
        r0, r1 = c.zeros(words), c.zeros(words)
        N.check(L.fkc_peer_set(c.handle, 2, 0, (ctypes.c_void_p * 2)(r0.ptr, r1.ptr)))
        c.set_wait_limit(100)
        d, k, n = 256, 128, 64
        w1 = c.to_device(O.normal(91, d * k, 0.0, 0.02).reshape(d, k))
        x = c.to_device(O.normal(92, k).reshape(1, k))
        # Rank 0's row-parallel GEMV: its partial rows into both regions,
        # counted in; rank 1's count in rank 0's region stays 0.
        c.launch("gemv_scatter", {"n": d, "k": k, "m": 1, "split": 1, "ldx": k, "xbuf": 1}, [w1, x])
        assert c.status() == 0
        w2 = c.to_device(O.normal(93, n * d, 0.0, 0.02).reshape(n, d))
        r = c.to_device(O.normal(94, d).reshape(1, d))
        g = c.to_device(O.uniform(95, d, 0.5, 1.5))
        xout, y = c.empty((1, d)), c.empty((1, n))
        c.set_wait_stats(True)
        t0 = time.perf_counter()
        c.launch("gemv_reduce_rmsnorm", {"n": n, "k": d, "m": 1, "split": 1, "ldr": d, "ldy": n, "eps": 1e-5,
                                         "factor": 1.0, "xbuf": 1}, [w2, r, g, xout, y])
        assert c.status() == 11
        assert time.perf_counter() - t0 < 1.0  # the default bound alone is about 2 s
        # Every block waited about the bound (SM cycles at the highest
        # clock: at least 100 us of device time, well under a second).
        ns, waits = c.read_wait_stats()
        c.set_wait_stats(False)
        assert 1 <= waits <= 2 * c.sms
        assert 90_000 <= ns / waits < 1e9, (ns, waits)
        assert c.read_wait_stats() == (0, 0)
        # Rank 0's own rows did arrive in its region (its count is d).
        flags = r0.download()[:8 * 3].view(np.uint32).reshape(3, 8)
        assert flags[1, 0] == d and flags[1, 1] == 0
        # The context still launches and reports a clean status.
        a, b, s = c.to_device(O.normal(96, 1024)), c.to_device(O.normal(97, 1024)), c.empty(1024)
        c.launch("add", {"n": 1024}, [a, b, s])
        assert same_bits(s.download(), O.add(O.normal(96, 1024), O.normal(97, 1024)))
        assert c.status() == 0
    finally:
        c.close()
