"""The oracle's routed-expert operations (test infrastructure), pinned to
the reference's meaning of Route, LinearRouted, GatedGelu and CombineRanks
(src/FuryKernel/Program/Eval.hs:291-320, 356-416, 648-659) and to its known
answer for a route (test/Test/FuryKernel/ProgramTest.hs:1500-1509)."""

import math

import numpy as np

from oracle import oracle as O


def test_route_known_answer():
    # evalRoute: the top 2 of [1, 3, 3, 2] are 1 and 2 (ties to the lower index), each half.
    ids, ws = O.route_topk(np.array([[1, 3, 3, 2]], np.float32), 2)
    assert ids.tolist() == [[1, 2]]
    assert ws.tolist() == [[0.5, 0.5]]


def test_route_orders_by_logit_then_index_and_weights_are_a_softmax():
    rng = np.random.default_rng(5)
    x = rng.standard_normal((7, 16)).astype(np.float32)
    x[3, [2, 9]] = 4.0  # a tie: the lower index first
    ids, ws = O.route_topk(x, 4)
    for r in range(7):
        order = sorted(range(16), key=lambda i: (-float(x[r, i]), i))[:4]
        assert ids[r].tolist() == order
        e = np.exp(x[r, order].astype(np.float64) - x[r, order[0]])
        assert np.allclose(ws[r], e / e.sum(), rtol=4e-7, atol=0)
    assert ids[3, :2].tolist() == [2, 9]
    scale = np.linspace(0.5, 2.0, 16).astype(np.float32)
    ids2, ws2 = O.route_topk(x, 4, scale)
    assert np.array_equal(ids2, ids)
    assert np.array_equal(ws2, (ws * scale[ids]).astype(np.float32))


def test_gelu_tanh_within_a_few_ulp_of_its_meaning():
    for v in np.linspace(-8, 8, 2001, dtype=np.float32):
        x = float(v)
        exact = 0.5 * x * (1 + math.tanh(math.sqrt(2 / math.pi) * (x + 0.044715 * x ** 3)))
        got = float(O.gelu_tanh(v))
        # A few roundings relative to the value, and tanh's own rounding carried
        # through 1 + tanh, which cancels where tanh nears -1: 0.5 |x| of it.
        eps = float(np.finfo(np.float32).eps)
        assert abs(got - exact) <= 4 * eps * abs(exact) + eps * 0.5 * abs(x), (x, got, exact)


def test_gemv_routed_is_the_gemv_of_each_rank_s_expert():
    rng = np.random.default_rng(6)
    entries, n, kk, m, k = 8, 24, 64, 3, 2
    table = rng.standard_normal((entries, n, kk)).astype(np.float32)
    ids = np.array([[3, 1], [1, 7], [0, 3]], np.uint32)
    shared = rng.standard_normal((m, kk)).astype(np.float32)
    per_rank = rng.standard_normal((m, k * kk)).astype(np.float32)
    for x, split in ((shared, 1), (per_rank, 2)):
        y = O.gemv_routed(table, ids, x, split)
        for r in range(m):
            for j in range(k):
                xs = x[r] if x.shape[1] == kk else x[r, j * kk:(j + 1) * kk]
                want = O.gemv(table[ids[r, j]], xs[None, :], split)[0]
                assert np.array_equal(y[r, j * n:(j + 1) * n].view(np.uint32), want.view(np.uint32))


def test_gated_gelu_and_combine_ranks():
    rng = np.random.default_rng(7)
    m, k, f, d = 2, 3, 8, 16
    gu = rng.standard_normal((m, k * 2 * f)).astype(np.float32)
    act = O.gated_gelu(gu, f)
    for r in range(m):
        for j in range(k):
            seg = gu[r, j * 2 * f:(j + 1) * 2 * f]
            want = np.array([np.float32(O.gelu_tanh(a)) * np.float32(b) for a, b in zip(seg[:f], seg[f:])],
                            np.float32)
            assert np.array_equal(act[r, j * f:(j + 1) * f], want)
    res = rng.standard_normal((m, d)).astype(np.float32)
    ws = rng.random((m, k)).astype(np.float32)
    segs = rng.standard_normal((m, k * d)).astype(np.float32)
    y = O.combine_ranks_add(res, ws, segs)
    for r in range(m):
        acc = ws[r, 0] * segs[r, :d]
        for j in range(1, k):
            acc = (acc + ws[r, j] * segs[r, j * d:(j + 1) * d]).astype(np.float32)
        assert np.array_equal(y[r], (res[r] + acc).astype(np.float32))
