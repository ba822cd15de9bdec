"""The oracle pinned against the reference's own known answers.

Each case restates a golden vector of the reference's test suite; the
oracle is trusted as a checker only because these hold.
"""

import math
import struct

import numpy as np
import pytest

from oracle import oracle as O


def f32(x):
    return np.float32(x)


def bits(x):
    return struct.unpack("<I", struct.pack("<f", float(x)))[0]


def test_splitmix_finaliser():
    # test/cpu/Cases.hs:886-892: mix(seed * 0x9E3779B97F4A7C15 + i), i from 1.
    def mix(z):
        m = (1 << 64) - 1
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & m
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & m
        return z ^ (z >> 31)

    for seed in (0, 7, 2026, 0xFFFFFFFFFFFFFFFF):
        for i in (1, 2, 1000):
            want = mix((seed * 0x9E3779B97F4A7C15 + i) & ((1 << 64) - 1))
            assert O.lib().fko_random(seed, i) == want


def test_cases_floats_stream():
    # Cases.hs:894-896 floats: (w >> 40) - 2^23 over 2^22, values in [-2, 2):
    # the same top 24 bits our U(a, b) uses. U(-2, 2) must reproduce it.
    seed = 61
    got = O.uniform(seed, 64, -2.0, 2.0)
    want = [((O.lib().fko_random(seed, i + 1) >> 40) - 2 ** 23) / 2 ** 22 for i in range(64)]
    assert np.array_equal(got, np.array(want, np.float32))


def test_simd_sum_pairwise_2_24_and_31_ones():
    # InterpTest.hs:50-55: 2^24 then 31 ones; pairwise only the first 1 rounds away.
    v = np.array([2.0 ** 24] + [1.0] * 31, np.float32)
    assert O.lib().fko_simd_sum(v, 32) == 16777246.0


def test_simd_sum_neighbours_first_lanes_16_17():
    # InterpTest.hs:56-62 and Cases.hs:515-526: 2^24 at lane 0, ones at 16, 17.
    v = np.zeros(32, np.float32)
    v[0] = 2.0 ** 24
    v[16] = v[17] = 1.0
    assert O.lib().fko_simd_sum(v, 32) == 16777218.0


def test_tg_reduce_sum_of_negative_zeros():
    # ReduceTest.hs:46-48: a sum of -0s is -0, of +0s +0.
    neg = np.full(256, -0.0, np.float32)
    pos = np.zeros(256, np.float32)
    assert bits(O.lib().fko_tg_reduce_sum(neg, 256)) == 0x80000000
    assert bits(O.lib().fko_tg_reduce_sum(pos, 256)) == 0x00000000


def test_tg_reduce_max_of_thread_indices():
    # ReduceTest.hs:44-45: the maximum over every thread's index is 255.
    lanes = np.arange(256, dtype=np.float32)
    assert O.lib().fko_tg_reduce_max(lanes, 256) == 255.0


def test_split_order_combine():
    # ReduceTest.hs:57-59: ((1e8 + 1) - 1e8) + 1 is 1 in f32; 3 + 4 + 5 + 6 = 18.
    # The GEMV's split combine (fko_gemv, split s) adds the partials in split
    # order; restated with one pack per split.
    # Virtual lane v = q * 32 + l takes pack v first, so pack 32 q is split q's
    # alone: k = 4 * 128, split q's one nonzero product at element 128 q.
    k = 512
    xk = np.zeros(k, np.float32)
    wk = np.zeros((1, k), np.float32)
    wk2 = np.zeros((1, k), np.float32)
    for q, (a, b) in enumerate(zip([1e8, 1.0, -1e8, 1.0], [3.0, 4.0, 5.0, 6.0])):
        xk[128 * q] = 1.0
        wk[0, 128 * q] = a
        wk2[0, 128 * q] = b
    assert O.gemv(wk, xk, split=4)[0, 0] == 1.0
    assert O.gemv(wk2, xk, split=4)[0, 0] == 18.0


def test_maximum_number_nan_and_zeros():
    # Cpu.hs:157-183 (pinned by Cases.hs:747-757): a NaN gives way, two NaNs
    # give the quiet NaN, +0 is above -0, -0 below +0 for the minimum.
    L = O.lib()
    nan = float("nan")
    assert L.fko_max(nan, 3.0) == 3.0
    assert L.fko_max(3.0, nan) == 3.0
    assert bits(L.fko_max(nan, nan)) == 0x7FC00000
    assert bits(L.fko_max(-0.0, 0.0)) == 0
    assert bits(L.fko_max(0.0, -0.0)) == 0
    assert bits(L.fko_min(-0.0, 0.0)) == 0x80000000


def test_transcendentals_binary64_rounded_once():
    # Cpu.hs:651-660: exp and rsqrt computed in binary64, rounded once.
    for v in (0.5, 1.0, 3.75, 1e-3, 88.0):
        assert O.lib().fko_exp.restype  # loaded
    from ctypes import c_float
    import ctypes

    L = O.lib()
    L.fko_exp.restype = ctypes.c_float
    L.fko_exp.argtypes = [ctypes.c_float]
    L.fko_rsqrt.restype = ctypes.c_float
    L.fko_rsqrt.argtypes = [ctypes.c_float]
    for v in (0.5, 1.0, 3.75, 1e-3, -20.0):
        assert L.fko_exp(v) == np.float32(math.exp(float(np.float32(v))))
    for v in (0.5, 2.0, 3.0, 1e-5):
        assert L.fko_rsqrt(v) == np.float32(1.0 / math.sqrt(float(np.float32(v))))


def test_reduce_tree_small_is_halving():
    x = O.uniform(2026, 256 * 4 + 17)
    p = O.reduce_partials(x)
    t = np.concatenate([x, np.full(256 * 5 - x.size, -0.0, np.float32)]).reshape(5, 256).copy()
    for s in (128, 64, 32, 16, 8, 4, 2, 1):
        t[:, :s] = t[:, :s] + t[:, s:2 * s]
    assert np.array_equal(p, t[:, 0])


def test_eval_small_known_answers():
    # Restating ProgramTest.hs evalSmall's shape of check: a linear layer of
    # exact small integers is exact, and its bound covers only flush terms.
    w = np.array([[1, 2], [3, 4]], np.float32)
    x = np.array([[5, 6]], np.float32)
    y, yb = O.r_linear(w, O.r_input(x))
    assert np.array_equal(y, [[17.0, 39.0]])
    assert np.all(yb < 1e-5)


def test_attention_over_one_position_returns_its_value():
    # ProgramTest.hs:1085-1106 (evalAttention): one position, its value back.
    d, heads = 8, 1
    length = 4
    kc = np.zeros((1, heads, length, d))
    vc = np.zeros((1, heads, length, d))
    kc[0, 0, 0] = np.arange(d)
    vc[0, 0, 0] = np.arange(d) * 0.5 - 1
    q = np.ones((1, d))
    y, yb = O.r_attend((q, np.zeros_like(q)), heads, 1, d, length, np.array([0], np.uint32),
                       np.array([0], np.uint32), kc, vc, 1.0 / math.sqrt(d))
    assert np.allclose(y[0], vc[0, 0, 0])


def _ulps_bf16(a, b):
    """Distance in bf16 steps, across zero too (ReduceTest.hs:91-96)."""
    def ordered(u):
        u = u.astype(np.int64)
        return np.where(u & 0x8000, -(u & 0x7FFF), u)
    return np.abs(ordered(a) - ordered(b))


@pytest.mark.parametrize("h", [64, 256, 1000, 4096])
def test_rmsnorm_within_one_bf16_ulp_of_its_f64_spec(h):
    """The reference's RMSNorm property (test/Test/FuryKernel/ReduceTest.hs:
    40-42, 96-107), for the f32 row kernel: its result, narrowed to bf16, is
    within one bf16 ulp of the f64 specification narrowed once; and a row's
    bits do not depend on the rows beside it (:109-119)."""
    rng = np.random.default_rng(h)
    rows = 3
    x = O.widen_bf16(O.narrow_bf16(rng.uniform(-8, 8, size=(rows, h)).astype(np.float32)))
    g = O.widen_bf16(O.narrow_bf16(rng.uniform(-2, 2, size=h).astype(np.float32)))
    eps = np.float32(1e-6)
    got = O.rmsnorm_rows(x, g, eps)
    d = x.astype(np.float64)
    s = 1.0 / np.sqrt((d * d).sum(axis=1, keepdims=True) / h + float(eps))
    spec = (d * s * g.astype(np.float64)).astype(np.float32)
    assert _ulps_bf16(O.narrow_bf16(got), O.narrow_bf16(spec)).max() <= 1
    alone = O.rmsnorm_rows(x[1:2], g, eps)
    assert np.array_equal(alone.view(np.uint32), got[1:2].view(np.uint32))


def test_gemm_tile_sums_k_in_order():
    """gemmTile's element sums k in order (Tile.hs:19-23), the fragment
    product adding a rounded product at a time (Cpu.hs:549-560): with
    1e8, 1, -1e8, 1 along k the in-order sum is 1 (pairwise would be 0 or
    2); and every element within the f64 evaluator's bound of A B^T
    (TileTest.hs:33-47)."""
    a = np.array([[1e8, 1.0, -1e8, 1.0] + [0.0] * 4], np.float32)
    b = np.ones((1, 8), np.float32)
    assert O.gemm_tile(a, b)[0, 0] == np.float32(1.0)
    rng = np.random.default_rng(5)
    A = rng.standard_normal((9, 96)).astype(np.float32)
    B = (0.02 * rng.standard_normal((7, 96))).astype(np.float32)
    got = O.gemm_tile(A, B)
    assert O.within(got, O.r_linear(B, O.r_input(A))).all()
