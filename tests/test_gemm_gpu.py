"""The prefill GEMMs on tcgen05 tensor cores (3xTF32) through the C ABI,
against the f64 evaluator: every element within its binary32 bound
(dotA, src/FuryKernel/Program/Eval.hs:747-754) and the normwise relative
error max|C - C64| / max|C64| <= 1e-4 (the path's GEMM tolerance). The
tensor cores sum in their own order, so no bit comparison with the CPU
target. gemm_tf32x3w (W split on the chip and held in tensor memory as the
MMA's A operand, the tile transposed, per-shape tile widths) forms the same
three products as gemm_tf32x3 from the same halves; it is held to the same
bounds, and to within 2^-14 of gemm_tf32x3's result (max |C - C0| /
max |C0|): with K whole it adds the products in gemm_tf32x3's order (the
same bits, measured), but where it splits K the two halves are separate
accumulations on the tensor cores, whose adds do not round to nearest, so
their sum drifts from the one long chain by up to about 2^-15 of max |C|
at K = 4096 (measured)."""

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    from furykernel_b200 import _native as N

    c = N.Context(0)
    yield c
    c.close()


def gemm(ctx, a, w):
    M, K = a.shape
    n = w.shape[0]
    da, dw = ctx.to_device(a), ctx.to_device(w)
    whi, wlo, ahi, alo = ctx.empty((n, K)), ctx.empty((n, K)), ctx.empty((M, K)), ctx.empty((M, K))
    dc = ctx.zeros((M, n))
    ctx.launch("split_tf32", {"n": n * K}, [dw, whi, wlo])
    ctx.launch("gemm_tf32x3", {"M": M, "N": n, "K": K, "ldc": n}, [da, ahi, alo, whi, wlo, dc])
    status = ctx.status()
    c = dc.download()
    hi, lo = whi.download(), wlo.download()
    for b in (da, dw, whi, wlo, ahi, alo, dc):
        b.free()
    return c, status, hi, lo


@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (256, 384, 512), (200, 300, 4096), (129, 130, 96),
                                   (512, 11008, 4096)])
def test_gemm_tf32x3_within_bounds(ctx, M, N, K):
    a = O.normal(3 + M, M * K).reshape(M, K)
    w = O.normal(4 + N, N * K, 0.0, 0.02).reshape(N, K)
    c, status, hi, lo = gemm(ctx, a, w)
    assert status == 0
    # The split: hi + lo represents w to within 2^-22 of |w|; both are TF32 values.
    assert np.all(np.abs(hi.astype(np.float64) + lo - w) <= np.abs(w) * 2.0 ** -21)
    assert np.all(hi.view(np.uint32) & 0x1FFF == 0) and np.all(lo.view(np.uint32) & 0x1FFF == 0)
    exact = a.astype(np.float64) @ w.astype(np.float64).T
    assert np.max(np.abs(c - exact)) / np.max(np.abs(exact)) <= 1e-4
    rows = np.arange(0, M, max(1, M // 4))[:4]  # the referee's bounds on a sample of rows
    ref = O.r_linear(w, O.r_input(a[rows]))
    assert O.within(c[rows], ref).all()


def gemm_w(ctx, a, w):
    M, K = a.shape
    n = w.shape[0]
    da, dw = ctx.to_device(a), ctx.to_device(w)
    ahi, alo = ctx.empty((M, K)), ctx.empty((M, K))
    dc = ctx.zeros((M, n))
    ctx.launch("gemm_tf32x3w", {"M": M, "N": n, "K": K, "ldc": n}, [da, ahi, alo, dw, dc])
    status = ctx.status()
    c = dc.download()
    for b in (da, dw, ahi, alo, dc):
        b.free()
    return c, status


# Shapes whose tiles (128 W rows x tm A rows, the launcher's pick on 148
# SMs) have tm 16, 96, 128, 160, 176 and 256: a 16-column accumulator to
# eight 32-column pieces, with and without a 16-column tail; ragged M and
# N; 3 and 4 ring stages.
@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (129, 130, 96), (512, 2752, 256), (511, 4096, 128),
                                   (640, 8192, 64), (512, 11008, 4096), (1024, 4096, 256), (1536, 11008, 128)])
def test_gemm_tf32x3w_within_bounds_and_as_split_kernel(ctx, M, N, K):
    a = O.normal(5 + M, M * K).reshape(M, K)
    w = O.normal(6 + N, N * K, 0.0, 0.02).reshape(N, K)
    c, status = gemm_w(ctx, a, w)
    assert status == 0
    exact = a.astype(np.float64) @ w.astype(np.float64).T
    assert np.max(np.abs(c - exact)) / np.max(np.abs(exact)) <= 1e-4
    rows = np.arange(0, M, max(1, M // 4))[:4]
    ref = O.r_linear(w, O.r_input(a[rows]))
    assert O.within(c[rows], ref).all()
    c0, status0, _, _ = gemm(ctx, a, w)
    assert status0 == 0
    assert np.max(np.abs(c.astype(np.float64) - c0)) <= np.max(np.abs(c0)) * 2.0 ** -14


# Tiles set by hand (fkc_set_gemm_tile): the widest tile with K whole, in
# two halves that add into C, and in equal shares over the SMs (a tile in
# two CTAs, pieces of any length); the narrowest and an odd width; a ragged
# shape (M, N not multiples of the tile, K a multiple of 16 but not of 32,
# an odd number of slabs), config 5's down projection and config 3c. Two
# parts of a tile add onto zero, the same bits in either order, so every
# tile gives the same bits run after run and is held to the same bounds.
@pytest.mark.parametrize("M,N,K,tm,parts", [(300, 1000, 4112, 256, 2), (300, 1000, 4112, 256, 1),
                                            (300, 1000, 4112, 16, 2), (300, 1000, 4112, 48, 1),
                                            (511, 4096, 11008, 256, 2), (64, 384, 48, 32, 2),
                                            (300, 4000, 4112, 16, 0), (512, 11008, 4096, 256, 0),
                                            (300, 1000, 4112, 32, 0)])
def test_gemm_tf32x3w_set_tiles(ctx, M, N, K, tm, parts):
    a = O.normal(7 + M, M * K).reshape(M, K)
    w = O.normal(8 + N, N * K, 0.0, 0.02).reshape(N, K)
    ctx.set_gemm_tile(tm, parts)
    try:
        c, status = gemm_w(ctx, a, w)
        c2, status2 = gemm_w(ctx, a, w)
    finally:
        ctx.set_gemm_tile(0)
    assert status == 0 and status2 == 0
    assert np.array_equal(c.view(np.uint32), c2.view(np.uint32))  # the same bits every run
    exact = a.astype(np.float64) @ w.astype(np.float64).T
    assert np.max(np.abs(c - exact)) / np.max(np.abs(exact)) <= 1e-4
    rows = np.arange(0, M, max(1, M // 4))[:4]
    ref = O.r_linear(w, O.r_input(a[rows]))
    assert O.within(c[rows], ref).all()


def test_split_tf32_vector_and_scalar_forms_agree(ctx):
    """split_tf32 over n a multiple of 4 (16-byte loads and stores) and over
    n + 1 (an element at a time): the same bits for the shared elements,
    each half a TF32 value and hi + lo within 2^-21 of x."""
    n = 1000
    x = O.normal(17, n + 1)
    dx = ctx.to_device(x)
    outs = []
    for m in (n, n + 1):
        hi, lo = ctx.empty(m), ctx.empty(m)
        ctx.launch("split_tf32", {"n": m}, [dx, hi, lo])
        outs.append((hi.download(), lo.download()))
        hi.free()
        lo.free()
    (h4, l4), (h1, l1) = outs
    assert np.array_equal(h4.view(np.uint32), h1[:n].view(np.uint32))
    assert np.array_equal(l4.view(np.uint32), l1[:n].view(np.uint32))
    assert np.all(h1.view(np.uint32) & 0x1FFF == 0) and np.all(l1.view(np.uint32) & 0x1FFF == 0)
    assert np.all(np.abs(h1.astype(np.float64) + l1 - x) <= np.abs(x) * 2.0 ** -21)
    dx.free()
