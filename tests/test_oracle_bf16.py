"""The oracle's restatement of the reference's bf16 GEMV family
(test/Test/FuryKernel/Gemv.hs), pinned by the reference's own properties
(test/Test/FuryKernel/GemvTest.hs): bit for bit with the exact sum where
f32 sums are exact (multiples of 1/8), within the bound of f32 accumulation
otherwise, a row's bits independent of the batch; and the conversions'
rounding (src/FuryKernel/Numerics.hs:33-48)."""

import numpy as np
import pytest

from oracle import oracle as O

RNG = np.random.default_rng(20261201)
VARIANTS = [(p, s) for p in (4, 8, 16) for s in (1, 2, 4)]


def bf16(a) -> np.ndarray:
    return O.narrow_bf16(np.asarray(a, np.float32))


def test_narrow_and_widen():
    ones = np.array([1.0, 1.00390625, 1.01171875, -2.0, 3.4e38, np.inf, -0.0], np.float32)
    # 1 + 2^-8 ties to even (down), 1 + 3 * 2^-8 ties to even (up), 3.4e38
    # rounds past bf16's largest finite value to infinity.
    assert bf16(ones).tolist() == [0x3F80, 0x3F80, 0x3F82, 0xC000, 0x7F80, 0x7F80, 0x8000]
    nan = np.array([0x7F800001], np.uint32).view(np.float32)
    assert int(bf16(nan)[0]) == 0x7FC0  # payload's high half kept, quiet bit set
    assert O.widen_bf16(np.array([0x7F81], np.uint16)).view(np.uint32)[0] == 0x7FC10000
    for v in (0x0001, 0x3F80, 0x8000, 0xFF80, 0x7F7F):
        b = np.array([v], np.uint16)
        assert int(bf16(O.widen_bf16(b))[0]) == v
        assert np.float32(O.lib().fko_widen_bf16(v)).view(np.uint32) == O.widen_bf16(b).view(np.uint32)[0]


def eighths(shape) -> np.ndarray:
    return bf16(RNG.integers(-8, 9, size=shape) / 8.0)


@pytest.mark.parametrize("pack,split", VARIANTS)
def test_exact_sums_give_the_spec_bit_for_bit(pack, split):
    for _ in range(4):
        n, m = int(RNG.integers(1, 9)), int(RNG.integers(1, 4))
        k = pack * int(RNG.integers(1, 49))
        w, x = eighths((n, k)), eighths((m, k))
        y = O.gemv_bf16(w, x, pack, split)
        exact = O.widen_bf16(x).astype(np.float64) @ O.widen_bf16(w).astype(np.float64).T
        assert np.array_equal(y, bf16(exact.astype(np.float32)))


@pytest.mark.parametrize("pack,split", VARIANTS)
def test_any_sums_within_the_bound_of_f32_accumulation(pack, split):
    n, m = 7, 3
    k = pack * 40
    w = bf16(RNG.uniform(-2, 2, size=(n, k)))
    x = bf16(RNG.uniform(-2, 2, size=(m, k)))
    got = O.widen_bf16(O.gemv_bf16(w, x, pack, split)).astype(np.float64)
    xw, ww = O.widen_bf16(x).astype(np.float64), O.widen_bf16(w).astype(np.float64)
    d = xw @ ww.T
    magnitude = np.abs(xw) @ np.abs(ww).T
    bound = 2.0 ** -8 * np.abs(d) + 2 * (k + 64) * 2.0 ** -24 * magnitude + 2.0 ** -126
    assert np.all(np.abs(got - d) <= bound)


@pytest.mark.parametrize("pack,split", VARIANTS)
def test_a_row_s_bits_do_not_depend_on_the_batch(pack, split):
    n, k = 5, pack * 33
    w = bf16(RNG.uniform(-2, 2, size=(n, k)))
    x = bf16(RNG.uniform(-2, 2, size=(6, k)))
    whole = O.gemv_bf16(w, x, pack, split)
    for i in range(6):
        assert np.array_equal(O.gemv_bf16(w, x[i:i + 1], pack, split)[0], whole[i])

