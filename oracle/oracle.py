"""TEST INFRASTRUCTURE -- the CPU oracle, not part of the product.

ctypes access to ``oracle/_build/libfko.so``: a C restatement of what the
reference's CPU target (src/FuryKernel/Cpu.hs) computes for this path's spec
kernels (``fko_*``) and of the f64 evaluator with its binary32 bounds
(src/FuryKernel/Program/Eval.hs, ``fkr_*``). Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline and reference
arms import this module, as the checker and as the timed CPU baseline; the
``furykernel_b200`` package never does.

Parity pins: the generator is the SplitMix finaliser of
test/cpu/Cases.hs:885-892; the reduction orders are pinned by the known
answers of test/Test/FuryKernel/InterpTest.hs:50-58 and ReduceTest.hs:46-59
(tests/test_oracle_pins.py). The reference itself cannot run here (no GHC,
no rustc), so no output of the reference pins this restatement beyond those.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libfko.so")
_lib = None

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_u64 = ctypes.c_uint64
_u32 = ctypes.c_uint32
_int = ctypes.c_int
_f32 = ctypes.c_float
_f64 = ctypes.c_double


def build() -> str:
    """Compile the restatement with its Makefile (strict IEEE flags)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        import fcntl

        sources = [os.path.join(_HERE, f) for f in ("fko_cpu.c", "fko_eval.c", "fko.h", "Makefile")]
        os.makedirs(os.path.dirname(_LIB_PATH), exist_ok=True)
        # One process builds at a time (ranks of a multi-process test start
        # together); the others find the library current when they get the lock.
        with open(_LIB_PATH + ".lock", "w") as lock:
            fcntl.flock(lock, fcntl.LOCK_EX)
            if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < max(map(os.path.getmtime, sources)):
                build()
        L = ctypes.CDLL(_LIB_PATH)
        sig = {
            "fko_random": (_u64, [_u64, _u64]),
            "fko_fill_uniform": (None, [_u64, _u64, _f64, _f64, _f32p]),
            "fko_fill_normal": (None, [_u64, _u64, _f64, _f64, _f32p]),
            "fko_fill_ints": (None, [_u64, _u64, _u32, _u32p]),
            "fko_max": (_f32, [_f32, _f32]),
            "fko_min": (_f32, [_f32, _f32]),
            "fko_simd_sum": (_f32, [_f32p, _int]),
            "fko_simd_max": (_f32, [_f32p, _int]),
            "fko_tg_reduce_sum": (_f32, [_f32p, _int]),
            "fko_tg_reduce_max": (_f32, [_f32p, _int]),
            "fko_reduce_pass1": (None, [_f32p, _u64, _f32p, _int]),
            "fko_reduce_pass2": (None, [_f32p, _u32, _f32p]),
            "fko_reduce_sum": (_f32, [_f32p, _u64, _int]),
            "fko_rmsnorm_rows": (None, [_f32p, _u32, _u32, ctypes.c_void_p, _f32, _f32, _f32p, _int]),
            "fko_softmax_rows": (None, [_f32p, _u32, _u32, _f32p, _int]),
            "fko_gemv": (None, [_f32p, _u32, _u32, _f32p, _u32, _u32, _f32p, _int]),
            "fko_gemv_bf16": (None, [_u16p, _u32, _u32, _u16p, _u32, _u32, _u32, _u16p, _int]),
            "fko_gemm_tile": (None, [_f32p, _u32, _u32, _f32p, _u32, _f32p, _int]),
            "fko_widen_bf16": (_f32, [ctypes.c_uint16]),
            "fko_narrow_bf16": (ctypes.c_uint16, [_f32]),
            "fko_widen_f16": (_f32, [ctypes.c_uint16]),
            "fko_narrow_f16": (ctypes.c_uint16, [_f32]),
            "fko_rope_tables": (None, [_f64, _u32, _u32, _u32, _f32p, _f32p]),
            "fko_rope": (None, [_f32p, _u32, _u32, _u32, _u32, _u32p, _f32p, _f32p, _f32p]),
            "fko_kv_store_ring": (None, [_f32p, _u32, _u32, _u32, _u32, _u32p, _u32p, _f32p]),
            "fko_attend_split": (None, [_f32p, _u32, _u32, _u32, _u32, _u32, _u32p, _u32p, _f32p, _f32p,
                                        _f32, _u32, _u32, _u32, _f32p, _f32p, _f32p, _int]),
            "fko_attend_combine": (None, [_u32, _u32, _u32, _u32p, _u32, _u32, _f32p, _f32p, _f32p, _f32p]),
            "fko_silu_mul": (None, [_f32p, _f32p, _u64, _f32p]),
            "fko_gelu_tanh": (ctypes.c_float, [_f32]),
            "fko_route_topk": (None, [_f32p, _u32, _u32, _u32, ctypes.c_void_p, _u32p, _f32p]),
            "fko_gemv_routed": (None, [_f32p, _u32, _u32, _u32, _u32p, _u32, _u32, _f32p, _u32, _u32, _f32p, _int]),
            "fko_gated_gelu": (None, [_f32p, _u64, _u32, _f32p]),
            "fko_combine_ranks_add": (None, [_f32p, _f32p, _f32p, _u32, _u32, _u32, _f32p]),
            "fko_add": (None, [_f32p, _f32p, _u64, _f32p]),
            "fko_gather": (None, [_f32p, _u32, _u32p, _u32, _f32, _f32p]),
            "fko_argmax": (None, [_f32p, _u32, _u32, _u32p]),
            "fkr_settle": (_f64, [_f64, _f64]),
            "fkr_widened": (_f64, [_f64]),
            "fkr_input": (None, [_f32p, _u64, _f64p, _f64p]),
            "fkr_linear": (None, [_f32p, _u32, _u32, _f64p, _f64p, _u32, _f64p, _f64p, _int]),
            "fkr_rmsnorm": (None, [_f64p, _f64p, _u32, _u32, _u32, ctypes.c_void_p, _f64, _f64, _f64p, _f64p]),
            "fkr_add": (None, [_f64p, _f64p, _f64p, _f64p, _u64, _f64p, _f64p]),
            "fkr_silu_mul": (None, [_f64p, _f64p, _f64p, _f64p, _u64, _f64p, _f64p]),
            "fkr_rope": (None, [_f64p, _f64p, _u32, _u32, _u32, _u32, _f64, _u32p, _f64p, _f64p]),
            "fkr_attend": (None, [_f64p, _f64p, _u32, _u32, _u32, _u32, _u32, _u32p, _u32p,
                                  _f64p, ctypes.c_void_p, _f64p, ctypes.c_void_p, _f64, _f64p, _f64p, _int]),
            "fkr_gather": (None, [_f32p, _u32, _u32p, _u32, _f64, _f64p, _f64p]),
            "fkr_argmax": (None, [_f64p, _f64p, _u32, _u32, _u32p, _i32p]),
            "fkr_softmax": (None, [_f64p, _f64p, _u32, _u32, _f64p, _f64p]),
            "fkr_sum": (None, [_f32p, _u64, ctypes.POINTER(_f64), ctypes.POINTER(_f64)]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def threads_default() -> int:
    return os.cpu_count() or 1


# ---------------------------------------------------------------------------
# Seeded inputs


def uniform(seed: int, n: int, a: float = -1.0, b: float = 1.0) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().fko_fill_uniform(seed, n, a, b, out)
    return out


def normal(seed: int, n: int, mu: float = 0.0, sigma: float = 1.0) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().fko_fill_normal(seed, n, mu, sigma, out)
    return out


def ints(seed: int, n: int, bound: int) -> np.ndarray:
    out = np.empty(n, np.uint32)
    lib().fko_fill_ints(seed, n, bound, out)
    return out


# ---------------------------------------------------------------------------
# Spec kernels, CPU-target semantics


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


def reduce_sum(x, threads: int = 1) -> np.float32:
    x = _c(x, np.float32)
    return np.float32(lib().fko_reduce_sum(x, x.size, threads))


def reduce_partials(x, threads: int = 1) -> np.ndarray:
    x = _c(x, np.float32)
    p = np.empty((x.size + 255) // 256, np.float32)
    lib().fko_reduce_pass1(x, x.size, p, threads)
    return p


def rmsnorm_rows(x, gamma, eps: float, factor: float = 1.0, threads: int = 1) -> np.ndarray:
    x = _c(x, np.float32)
    rows, h = x.shape
    y = np.empty_like(x)
    g = None if gamma is None else _c(gamma, np.float32)
    lib().fko_rmsnorm_rows(x, rows, h, None if g is None else g.ctypes.data, eps, factor, y, threads)
    return y


def softmax_rows(x, threads: int = 1) -> np.ndarray:
    x = _c(x, np.float32)
    y = np.empty_like(x)
    lib().fko_softmax_rows(x, x.shape[0], x.shape[1], y, threads)
    return y


def gemv(w, x, split: int = 1, threads: int = 1) -> np.ndarray:
    w = _c(w, np.float32)
    x = _c(x, np.float32)
    n, k = w.shape
    x2 = x.reshape(-1, k)
    y = np.empty((x2.shape[0], n), np.float32)
    lib().fko_gemv(w, n, k, x2, x2.shape[0], split, y, threads)
    return y


def gemm_tile(a, b, threads: int = 1) -> np.ndarray:
    """C = A B^T as the CPU target's gemmTile sums it (k in order)."""
    a = _c(a, np.float32)
    b = _c(b, np.float32)
    M, K = a.shape
    N = b.shape[0]
    c = np.empty((M, N), np.float32)
    lib().fko_gemm_tile(a, M, K, b, N, c, threads)
    return c


def gemv_bf16(w, x, pack: int = 8, split: int = 1, threads: int = 1) -> np.ndarray:
    """The reference's bf16 GEMV family (test/Test/FuryKernel/Gemv.hs):
    w [n, k] and x [m, k] as bf16 bits (uint16), y [m, n] bf16 bits."""
    w = _c(w, np.uint16)
    x = _c(x, np.uint16)
    n, k = w.shape
    x2 = x.reshape(-1, k)
    y = np.empty((x2.shape[0], n), np.uint16)
    lib().fko_gemv_bf16(w, n, k, x2, x2.shape[0], pack, split, y, threads)
    return y


def narrow_bf16(a) -> np.ndarray:
    """binary32 -> bf16 bits, round to nearest even, NaN quieted
    (narrowBF16, src/FuryKernel/Numerics.hs:41-48), vectorised."""
    a = np.ascontiguousarray(a, np.float32)
    w = a.view(np.uint32).astype(np.uint64)
    lsb = (w >> 16) & 1
    out = ((w + 0x7FFF + lsb) >> 16).astype(np.uint16)
    nan = np.isnan(a)
    out[nan] = ((w[nan] >> 16) | 0x0040).astype(np.uint16)
    return out


def widen_bf16(b) -> np.ndarray:
    """bf16 bits -> binary32, exact, NaN quieted (widenBF16,
    Numerics.hs:33-38), vectorised."""
    w = np.ascontiguousarray(b, np.uint16).astype(np.uint32) << 16
    nan = ((w & 0x7F800000) == 0x7F800000) & ((w & 0x007FFFFF) != 0)
    w[nan] |= 0x00400000
    return w.view(np.float32)


def narrow_f16(a) -> np.ndarray:
    """binary32 -> binary16 bits: nearest, ties to even, gradual underflow,
    half an ulp past the largest finite value or more to infinity, a NaN
    quiet with its sign and top payload bits (narrowF16,
    src/FuryKernel/Numerics.hs:100-130), vectorised on the bits."""
    a = np.ascontiguousarray(a, np.float32)
    w = a.view(np.uint32).astype(np.int64)
    sign = (w >> 16) & 0x8000
    e = (w >> 23) & 0xFF
    m = w & 0x7FFFFF
    unbiased = e - 127

    def round_even(kept, rest, half):
        return kept + ((rest > half) | ((rest == half) & ((kept & 1) == 1)))

    out = np.zeros(a.shape, np.int64)
    normal = (unbiased >= -14) & (unbiased < 16) & (e != 0xFF)
    out[normal] = round_even(((unbiased[normal] + 15) << 10) | (m[normal] >> 13), m[normal] & 0x1FFF, 0x1000)
    shift = -(unbiased + 1)
    sub = (unbiased < -14) & (e != 0) & (shift <= 24)
    full = m[sub] | 0x800000
    s = shift[sub]
    out[sub] = round_even(full >> s, full & ((1 << s) - 1), 1 << (s - 1))
    out[(unbiased >= 16) & (e != 0xFF)] = 0x7C00
    out[(e == 0xFF) & (m == 0)] = 0x7C00
    nan = (e == 0xFF) & (m != 0)
    out[nan] = 0x7E00 | (m[nan] >> 13)
    return (out | sign).astype(np.uint16)


def widen_f16(h) -> np.ndarray:
    """binary16 bits -> binary32, exact, a NaN quiet with its sign and
    payload (widenF16, src/FuryKernel/Numerics.hs:51-66), vectorised."""
    h = np.ascontiguousarray(h, np.uint16)
    out = h.view(np.float16).astype(np.float32)
    bits = h.astype(np.uint32)
    nan = ((bits & 0x7C00) == 0x7C00) & ((bits & 0x3FF) != 0)
    ov = out.view(np.uint32)
    ov[nan] = ((bits[nan] & 0x8000) << 16) | 0x7FC00000 | ((bits[nan] & 0x3FF) << 13)
    return out


def _round_to_grid(x, lowest: int, digits: int, overflow: float):
    """binary64 values rounded once, to nearest with ties to even, to a
    format whose significands have `digits` bits after the leading one and
    whose exponents go down to `lowest` (gradual underflow below it); a
    rounded magnitude at or past `overflow` is infinity. NaNs, infinities
    and zeros are kept."""
    x = np.asarray(x, np.float64)
    out = x.copy()
    ok = np.isfinite(x) & (x != 0)
    _, exp = np.frexp(x[ok])
    e = np.maximum(exp - 1, lowest)  # the leading bit's exponent, floored at the normal range
    ulp = np.ldexp(1.0, e - digits)
    rounded = np.rint(x[ok] / ulp) * ulp  # exact scalings; rint ties to even
    rounded[np.abs(rounded) >= overflow] = np.copysign(np.inf, rounded[np.abs(rounded) >= overflow])
    out[ok] = rounded
    return out


def narrow_f16_f64(x) -> np.ndarray:
    """binary64 -> binary16 bits in one rounding, not through binary32
    (narrowF16Double, src/FuryKernel/Numerics.hs:132-155): nearest, ties to
    even, gradual underflow, overflow to infinity, the sign of zero kept, a
    NaN quiet with its sign and top payload bits."""
    x = np.asarray(x, np.float64)
    with np.errstate(over="ignore"):
        bits = _round_to_grid(x, -14, 10, 65536.0).astype(np.float16).view(np.uint16)
    w = x.view(np.uint64)
    nan = np.isnan(x)
    bits[nan] = (((w[nan] >> 48) & 0x8000) | 0x7E00 | ((w[nan] >> 42) & 0x1FF)).astype(np.uint16)
    return bits


def round_bf16_f64(x) -> np.ndarray:
    """binary64 values rounded once to bfloat16's values, as binary64
    (roundBF16, src/FuryKernel/Program/Eval.hs:669-682): nearest, ties to
    even, the exponent floored at -126, a magnitude of 2^128 or more
    infinity."""
    return _round_to_grid(x, -126, 7, 2.0 ** 128)


def round_to(t: str, x) -> np.ndarray:
    """binary64 values rounded to a cache's element type, directly from the
    binary64 (roundTo, src/FuryKernel/Program/Eval.hs:930-934)."""
    if t == "bf16":
        return round_bf16_f64(x)
    if t == "f16":
        return widen_f16(narrow_f16_f64(x)).astype(np.float64)
    raise ValueError(f"no rounding to {t}")


def rope_tables(theta: float, d: int, rotated: int, positions: int):
    c = np.empty((positions, rotated), np.float32)
    s = np.empty((positions, rotated), np.float32)
    lib().fko_rope_tables(theta, d, rotated, positions, c, s)
    return c, s


def rope(x, heads: int, d: int, rotated: int, pos, cos_t, sin_t) -> np.ndarray:
    x = _c(x, np.float32)
    m = x.shape[0]
    y = np.empty_like(x)
    lib().fko_rope(x, m, heads, d, rotated, _c(pos, np.uint32), _c(cos_t, np.float32), _c(sin_t, np.float32), y)
    return y


def kv_store_ring(x, kv_heads: int, d: int, length: int, pos, slot, cache: np.ndarray) -> None:
    x = _c(x, np.float32)
    assert cache.dtype == np.float32 and cache.flags.c_contiguous
    lib().fko_kv_store_ring(x, x.shape[0], kv_heads, d, length, _c(pos, np.uint32), _c(slot, np.uint32), cache)


def attend(q, heads, kv_heads, d, length, pos, slot, kc, vc, scale, chunk, warps, max_splits, threads=1):
    """Split attention then its combine, the CUDA kernels' order."""
    q = _c(q, np.float32)
    m = q.shape[0]
    pos = _c(pos, np.uint32)
    slot = _c(slot, np.uint32)
    pm = np.zeros(m * heads * max_splits, np.float32)
    pl = np.zeros(m * heads * max_splits, np.float32)
    pa = np.zeros(m * heads * max_splits * d, np.float32)
    lib().fko_attend_split(q, m, heads, kv_heads, d, length, pos, slot, _c(kc, np.float32), _c(vc, np.float32),
                           scale, chunk, warps, max_splits, pm, pl, pa, threads)
    out = np.empty((m, heads * d), np.float32)
    lib().fko_attend_combine(m, heads, d, pos, chunk, max_splits, pm, pl, pa, out)
    return out, (pm, pl, pa)


def silu_mul(a, b) -> np.ndarray:
    a = _c(a, np.float32)
    y = np.empty_like(a)
    lib().fko_silu_mul(a, _c(b, np.float32), a.size, y)
    return y


def gelu_tanh(x: float) -> np.float32:
    """GELU, the tanh form, in this target's binary32 order (fko_gelu_tanh)."""
    return np.float32(lib().fko_gelu_tanh(float(x)))


def route_topk(x, k: int, scale=None):
    """Each row's top k ids (ties to the lower index) and their softmax
    weights (routeRow, Eval.hs:648-656), times the expert scale if given."""
    x = _c(x, np.float32)
    m, n = x.reshape(-1, x.shape[-1]).shape
    ids = np.empty((m, k), np.uint32)
    ws = np.empty((m, k), np.float32)
    sc = _c(scale, np.float32) if scale is not None else None
    lib().fko_route_topk(x, m, n, k, sc.ctypes.data if sc is not None else None, ids, ws)
    return ids, ws


def gemv_routed(table, ids, x, split: int = 1, threads: int = 1) -> np.ndarray:
    """LinearRouted: table [entries, n, kk], ids [m, k], x [m, kk] (every
    rank's input) or [m, k * kk] (a segment a rank); y [m, k * n]."""
    table = _c(table, np.float32)
    entries, n, kk = table.shape
    ids = _c(ids, np.uint32)
    m, k = ids.shape
    x = _c(x, np.float32).reshape(m, -1)
    y = np.empty((m, k * n), np.float32)
    lib().fko_gemv_routed(table, entries, n, kk, ids, m, k, x, x.shape[1], split, y, threads)
    return y


def gated_gelu(x, f: int) -> np.ndarray:
    """GatedGelu of segments of 2 f: gelu(first half) * second half."""
    x = _c(x, np.float32)
    segs = x.size // (2 * f)
    y = np.empty(segs * f, np.float32)
    lib().fko_gated_gelu(x, segs, f, y)
    return y.reshape(x.shape[:-1] + (x.shape[-1] // 2,)) if x.ndim > 1 else y


def combine_ranks_add(r, ws, segs) -> np.ndarray:
    """r + the route-weighted sum of the ranks' segments, in rank order."""
    r = _c(r, np.float32)
    ws = _c(ws, np.float32)
    m, k = ws.shape
    d = r.shape[-1]
    y = np.empty((m, d), np.float32)
    lib().fko_combine_ranks_add(r, ws, _c(segs, np.float32), m, k, d, y)
    return y


def add(a, b) -> np.ndarray:
    a = _c(a, np.float32)
    y = np.empty_like(a)
    lib().fko_add(a, _c(b, np.float32), a.size, y)
    return y


def gather(table, tokens, factor: float = 1.0) -> np.ndarray:
    table = _c(table, np.float32)
    tokens = _c(tokens, np.uint32)
    width = table.shape[1]
    y = np.empty((tokens.size, width), np.float32)
    lib().fko_gather(table, width, tokens, tokens.size, factor, y)
    return y


def argmax(x) -> np.ndarray:
    x = _c(x, np.float32)
    m, n = x.shape
    ids = np.empty(m, np.uint32)
    lib().fko_argmax(x, m, n, ids)
    return ids


# ---------------------------------------------------------------------------
# The f64 referee: (values, bounds) pairs


def r_input(x):
    x = _c(x, np.float32)
    v = np.empty(x.shape, np.float64)
    b = np.empty(x.shape, np.float64)
    lib().fkr_input(x, x.size, v, b)
    return v, b


def r_linear(w, xv, threads: int = 0):
    w = _c(w, np.float32)
    x, xb = (_c(a, np.float64) for a in xv)
    n, k = w.shape
    m = x.size // k
    y = np.empty((m, n), np.float64)
    yb = np.empty((m, n), np.float64)
    lib().fkr_linear(w, n, k, x, xb, m, y, yb, threads or threads_default())
    return y, yb


def r_rmsnorm(xv, seg: int, gamma, eps: float, factor: float = 1.0):
    x, xb = (_c(a, np.float64) for a in xv)
    m, width = x.shape
    y = np.empty_like(x)
    yb = np.empty_like(x)
    g = None if gamma is None else _c(gamma, np.float32)
    lib().fkr_rmsnorm(x, xb, m, width, seg, None if g is None else g.ctypes.data, eps, factor, y, yb)
    return y, yb


def r_add(av, cv):
    a, ab = (_c(t, np.float64) for t in av)
    c, cb = (_c(t, np.float64) for t in cv)
    y = np.empty_like(a)
    yb = np.empty_like(a)
    lib().fkr_add(a, ab, c, cb, a.size, y, yb)
    return y, yb


def r_silu_mul(av, cv):
    a, ab = (_c(t, np.float64) for t in av)
    c, cb = (_c(t, np.float64) for t in cv)
    y = np.empty_like(a)
    yb = np.empty_like(a)
    lib().fkr_silu_mul(a, ab, c, cb, a.size, y, yb)
    return y, yb


def r_rope(xv, d: int, rotated: int, theta: float, pos):
    x, xb = (_c(t, np.float64) for t in xv)
    m, width = x.shape
    y = np.empty_like(x)
    yb = np.empty_like(x)
    lib().fkr_rope(x, xb, m, width, d, rotated, theta, _c(pos, np.uint32), y, yb)
    return y, yb


def r_attend(qv, heads, kv_heads, d, length, pos, slot, kc, vc, scale, kcb=None, vcb=None, threads: int = 0):
    q, qb = (_c(t, np.float64) for t in qv)
    m = q.shape[0]
    kc = _c(kc, np.float64)
    vc = _c(vc, np.float64)
    kcb = None if kcb is None else _c(kcb, np.float64)
    vcb = None if vcb is None else _c(vcb, np.float64)
    y = np.empty((m, heads * d), np.float64)
    yb = np.empty((m, heads * d), np.float64)
    lib().fkr_attend(q, qb, m, heads, kv_heads, d, length, _c(pos, np.uint32), _c(slot, np.uint32),
                     kc, None if kcb is None else kcb.ctypes.data, vc, None if vcb is None else vcb.ctypes.data,
                     scale, y, yb, threads or threads_default())
    return y, yb


def r_gather(table, tokens, factor: float = 1.0):
    table = _c(table, np.float32)
    tokens = _c(tokens, np.uint32)
    width = table.shape[1]
    y = np.empty((tokens.size, width), np.float64)
    yb = np.empty((tokens.size, width), np.float64)
    lib().fkr_gather(table, width, tokens, tokens.size, factor, y, yb)
    return y, yb


def r_argmax(xv):
    x, xb = (_c(t, np.float64) for t in xv)
    m, n = x.shape
    ids = np.empty(m, np.uint32)
    dec = np.empty(m, np.int32)
    lib().fkr_argmax(x, xb, m, n, ids, dec)
    return ids, dec.astype(bool)


def r_softmax(xv):
    x, xb = (_c(t, np.float64) for t in xv)
    m, n = x.shape
    y = np.empty_like(x)
    yb = np.empty_like(x)
    lib().fkr_softmax(x, xb, m, n, y, yb)
    return y, yb


def r_sum(x):
    x = _c(x, np.float32)
    y = _f64()
    yb = _f64()
    lib().fkr_sum(x, x.size, ctypes.byref(y), ctypes.byref(yb))
    return y.value, yb.value


def widened(b):
    return b * (1.0 + 2.0 ** -20)


def within(got, exact_bound) -> np.ndarray:
    """Elementwise: got lies within the widened bound of the exact value
    (the comparison of Eval.hs:940-944, for binary32 values)."""
    v, b = exact_bound
    got = np.asarray(got, np.float64)
    return (np.abs(got - v) <= widened(b)) | (np.isnan(got) & np.isnan(v)) | np.isinf(b)
