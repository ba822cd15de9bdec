"""The oracle's binary16 conversions, pinned by the reference's own tests of
them (test/Test/FuryKernel/NumericsTest.hs:27-51, :77-78, :118-119,
:127-148): the known answers, the round trip of every binary16 value, every
midpoint between neighbouring finite values, and nearest-rounding of random
binary32 values. The C restatement (fko_widen_f16, fko_narrow_f16) and the
vectorised one (widen_f16, narrow_f16) are held to each other as well."""

import numpy as np

from oracle import oracle as O


def f32(bits) -> np.ndarray:
    return np.asarray(bits, np.uint32).view(np.float32)


def bits32(a) -> np.ndarray:
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def narrow_c(a) -> np.ndarray:
    return np.array([O.lib().fko_narrow_f16(float(v)) for v in np.asarray(a, np.float32).ravel()], np.uint16)


def widen_c(h) -> np.ndarray:
    return np.array([O.lib().fko_widen_f16(int(v)) for v in np.asarray(h, np.uint16).ravel()], np.float32)


def test_known_answers():
    # NumericsTest.hs:45-51: the largest finite value, half an ulp short of
    # it and past it, the smallest subnormal, half of it (a tie to 0), 1.5
    # of it (a tie to 2), negative zero.
    xs = np.array([65504, 65519.996, 65520, 2.0 ** -24, 2.0 ** -25, 1.5 * 2.0 ** -24, -0.0], np.float32)
    want = [0x7BFF, 0x7BFF, 0x7C00, 0x0001, 0x0000, 0x0002, 0x8000]
    assert O.narrow_f16(xs).tolist() == want
    assert narrow_c(xs).tolist() == want
    # :73: 1 + 2^-11 + 2^-30, rounded to binary32 first, is the tie 1 + 2^-11.
    assert int(O.narrow_f16(np.array([1 + 2.0 ** -11 + 2.0 ** -30], np.float32))[0]) == 0x3C00


def test_nans():
    # :28-34: a NaN narrows to a quiet NaN of the same sign.
    nan = f32([0xFF800001])
    for h in (int(O.narrow_f16(nan)[0]), int(narrow_c(nan)[0])):
        assert h & 0x8200 == 0x8200 and h & 0x7C00 == 0x7C00 and h & 0x3FF
    # :40-43: NaNs widen quiet, their sign and payload kept; infinities stay.
    hs = np.array([0x7C01, 0xFD00, 0x7E01, 0xFC00], np.uint16)
    want = [0x7FC02000, 0xFFE00000, 0x7FC02000, 0xFF800000]
    assert bits32(O.widen_f16(hs)).tolist() == want
    assert bits32(widen_c(hs)).tolist() == want


def test_every_value_round_trips_and_both_restatements_agree():
    # :27-28: binary16 -> binary32 -> binary16 is the identity, NaNs aside.
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    w = O.widen_f16(h)
    nan = np.isnan(w)
    assert int(nan.sum()) == 2 * 1023
    back = O.narrow_f16(w)
    assert np.array_equal(back[~nan], h[~nan])
    assert np.array_equal(bits32(w), bits32(widen_c(h)))
    assert np.array_equal(back, narrow_c(w))
    # Widening is exact: numpy's binary16 values, NaNs aside.
    assert np.array_equal(w[~nan], h.view(np.float16)[~nan].astype(np.float32))


def test_every_midpoint_ties_to_even_and_its_neighbours_go_to_the_nearer():
    # :77-78, :127-148: neighbours lo, lo + 1 up to the largest finite value,
    # and their negations.
    lo = np.arange(0, 0x7BFF, dtype=np.uint32).astype(np.uint16)
    hi = (lo.astype(np.uint32) + 1).astype(np.uint16)
    a, b = O.widen_f16(lo), O.widen_f16(hi)
    mid = (a + (b - a) / np.float32(2)).astype(np.float32)
    above = f32(bits32(mid) + 1)
    below = f32(bits32(mid) - 1)
    even = np.where(lo % 2 == 0, lo, hi)
    for sign in (1, -1):
        flip = 0x8000 if sign < 0 else 0
        for x, want in ((mid, even), (above, hi), (below, lo)):
            got = O.narrow_f16((sign * x).astype(np.float32))
            assert np.array_equal(got, (want.astype(np.uint32) | flip).astype(np.uint16))
            assert np.array_equal(narrow_c((sign * x[::97]).astype(np.float32)),
                                  (want[::97].astype(np.uint32) | flip).astype(np.uint16))


def test_random_values_round_to_the_nearest():
    # :118-119: narrowing rounds to nearest, ties to even, within +-65536;
    # numpy's own binary16 conversion is a third statement of the rule.
    rng = np.random.default_rng(20261202)
    xs = np.concatenate([rng.uniform(-65536, 65536, 20000), rng.standard_normal(20000) * 2.0 ** -14,
                         rng.standard_normal(20000) * 0.02]).astype(np.float32)
    got = O.narrow_f16(xs)
    with np.errstate(over="ignore"):  # past 65520 numpy's conversion overflows to infinity too
        assert np.array_equal(got, xs.astype(np.float16).view(np.uint16))
    finite = np.abs(xs) < 65520
    v = O.widen_f16(got[finite]).astype(np.float64)
    err = np.abs(v - xs[finite].astype(np.float64))
    # The ulp of the result's binade (subnormals: 2^-24).
    ulp = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(v), 2.0 ** -14))) - 10)
    assert np.all(err <= ulp / 2)
    assert np.array_equal(narrow_c(xs[::50]), got[::50])


def test_binary64_narrows_once():
    # NumericsTest.hs:82-96: narrowF16Double's known answers.
    xs = np.array([65504, 65519.99999999999, 65520, -1e300, 2.0 ** -24, 2.0 ** -25, 2.0 ** -25 + 2.0 ** -60,
                   -(2.0 ** -26), 5e-324, -0.0, np.inf, 1 + 2.0 ** -11 + 2.0 ** -25], np.float64)
    want = [0x7BFF, 0x7BFF, 0x7C00, 0xFC00, 0x0001, 0x0000, 0x0001, 0x8000, 0x0000, 0x8000, 0x7C00, 0x3C01]
    assert O.narrow_f16_f64(xs).tolist() == want
    nan = np.array([0xFFF0000000000001], np.uint64).view(np.float64)
    assert int(O.narrow_f16_f64(nan)[0]) & 0xFE00 == 0xFE00
    # Through binary32 the same value rounds twice, to the tie and then even.
    assert int(O.narrow_f16(np.array([1 + 2.0 ** -11 + 2.0 ** -25], np.float32))[0]) == 0x3C00


def test_binary64_narrowing_is_the_nearest_value():
    # NumericsTest.hs:98-104: binary64 narrows to the binary16 a rational
    # would; here: the nearest of the neighbouring binary16 values, exactly,
    # ties to the even one.
    from fractions import Fraction

    rng = np.random.default_rng(7)
    xs = np.concatenate([rng.uniform(-70000, 70000, 300), rng.standard_normal(300) * 2.0 ** -16,
                         rng.standard_normal(300)])
    got = O.narrow_f16_f64(xs)
    values = O.widen_f16(np.arange(0x7C00, dtype=np.uint32).astype(np.uint16)).astype(np.float64)
    for x, h in zip(xs.tolist(), got.tolist()):
        a = abs(x)
        if a >= 65520:
            assert h & 0x7FFF == 0x7C00
            continue
        i = int(np.searchsorted(values, a, side="right")) - 1
        lo = i
        hi = min(i + 1, 0x7BFF)
        dlo, dhi = abs(Fraction(a) - Fraction(values[lo])), abs(Fraction(values[hi]) - Fraction(a))
        want = lo if dlo < dhi or (dlo == dhi and lo % 2 == 0) else hi
        assert h & 0x7FFF == want and (h >> 15) == (x < 0)


def test_bf16_rounding_from_binary64():
    # roundBF16 (Eval.hs:669-682) against narrowBF16 where binary32 holds the
    # value exactly, and at a double-rounding case it does not.
    rng = np.random.default_rng(8)
    xs = rng.standard_normal(5000).astype(np.float32)
    assert np.array_equal(O.round_bf16_f64(xs.astype(np.float64)),
                          O.widen_bf16(O.narrow_bf16(xs)).astype(np.float64))
    x = 1 + 2.0 ** -8 + 2.0 ** -40  # past the tie: up, where binary32 would round to the tie and then down
    assert O.round_bf16_f64(np.array([x]))[0] == 1 + 2.0 ** -7
    assert O.round_bf16_f64(np.array([3.4e38, -3.5e38, 2.0 ** -133, 2.0 ** -134]))[:2].tolist() == [np.inf, -np.inf]
    assert O.round_bf16_f64(np.array([2.0 ** -133, 2.0 ** -134, 1.5 * 2.0 ** -133])).tolist() == \
        [2.0 ** -133, 0.0, 2.0 ** -132]


def test_stores_are_judged_in_the_cache_type():
    # ProgramTest.hs:1190-1199: a one-element dot of 1 and 0.1 stored into a
    # cache of one element: an f16 cache keeps f16's 0.1 and refuses bf16's,
    # a bf16 cache the other way round.
    from tests.model_check import may_store

    exact = np.array([float(np.float32(0.1))])
    bound = exact * 2.0 ** -24
    f16_tenth, bf16_tenth = np.array([0.0999755859375]), np.array([0.10009765625])
    assert may_store("f16", exact, bound, f16_tenth)
    assert not may_store("f16", exact, bound, bf16_tenth)
    assert may_store("bf16", exact, bound, bf16_tenth)
    assert not may_store("bf16", exact, bound, f16_tenth)
    # Unbounded: anything; a NaN exact value: only a NaN.
    assert may_store("f16", exact, np.array([np.inf]), np.array([7.0]))
    assert may_store("bf16", np.array([np.nan]), bound, np.array([np.nan]))
    assert not may_store("bf16", np.array([np.nan]), bound, np.array([1.0]))
