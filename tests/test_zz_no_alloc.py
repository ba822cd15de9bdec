"""The reduction entry point that allocates nothing (fkc_reduce_sum_f32_noalloc),
for callers that cannot call cudaMalloc: called through the C ABI, its
output must be the bits of the table's reduce_groups + reduce_final on the
same input, and of the oracle's restatement of the CPU target's order, on
two calls in a row (the second after the first has left its scratch
behind), and a size past its static scratch must be refused.

Kept in a file that pytest collects last, so that a run that stops at its
first failure has run every other test first."""

import ctypes

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


def noalloc_fn():
    from furykernel_b200 import _native as N

    fn = N.lib().fkc_reduce_sum_f32_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p]
    return fn


def table_sum(ctx, xd, n):
    groups = (n + 255) // 256
    part = ctx.empty(groups)
    y = ctx.empty(1)
    ctx.launch("reduce_groups", {"n": n}, [xd, part])
    ctx.launch("reduce_final", {"count": groups}, [part, y])
    out = y.download()[0]
    part.free()
    y.free()
    return out


def test_noalloc_sum_matches_the_table_kernels_twice(ctx):
    from furykernel_b200 import _native as N

    fn = noalloc_fn()
    stream = ctx.stream()
    for n, seed in ((16_777_216, 31), (1_000_003, 32)):
        x = O.uniform(seed, n, -1.0, 1.0)
        xd = ctx.to_device(x)
        yd = ctx.empty(1)
        assert fn(xd.ptr, n, yd.ptr, stream) == N.FKC_OK, N.lib().fkc_last_error().decode()
        ctx.sync()
        got = yd.download()[0]
        want = table_sum(ctx, xd, n)
        assert np.float32(got).view(np.uint32) == np.float32(want).view(np.uint32), (n, got, want)
        # And the CPU target's order, restated by the oracle, bit for bit.
        ref = O.reduce_sum(x, O.threads_default())
        assert np.float32(got).view(np.uint32) == np.float32(ref).view(np.uint32), (n, got, ref)
        xd.free()
        yd.free()


def test_noalloc_sum_refuses_past_its_scratch(ctx):
    from furykernel_b200 import _native as N

    fn = noalloc_fn()
    yd = ctx.empty(1)
    rc = fn(yd.ptr, (1 << 26) + 1, yd.ptr, ctx.stream())
    assert rc == N.FKC_ERR_ARGUMENT
    assert "outside 1..67108864" in N.lib().fkc_last_error().decode()
    yd.free()
