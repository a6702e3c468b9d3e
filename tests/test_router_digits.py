"""Integer model of the tensor-core router's digit planes (CPU, exact).

router_digits_kernel (mlx-rs_b200/csrc/router_tc.cu) writes each row as an
integer row X (|X| < 2^30) times 2^u and splits every X into four balanced
base-256 digits with (X + 0x808080) ^ 0x808080, byte 3 - k being digit k.
router_tc_kernel sums the 16 plane products sum_i dx_k[i] dw_l[i] into 7 sums
by weight 2^(8 (6 - k - l)); its split-K form keeps only the 13 products with
k + l <= 4 and bounds the other three by D (2^23 + 2^14)
(logit_from_digit_sums in mlx-rs_b200/csrc/exact_dot.cuh). These tests check
that arithmetic with Python integers: the split reconstructs X, 16 products
give the exact integer dot product, and the three dropped ones stay within
the bound, which the worst case reaches.
"""
import numpy as np
import pytest


def digits(X):
    """The four balanced digits of X as the kernel forms them (k = 0 is the top)."""
    o = ((int(X) + 0x808080) & 0xFFFFFFFF) ^ 0x808080
    out = []
    for k in range(4):
        b = (o >> (8 * (3 - k))) & 0xFF
        out.append(b - 256 if b >= 128 else b)
    return out


def plane_sums(xd, wd, nsums):
    """Digit sums A[g] = sum over k + l = g (g < nsums) of sum_i dx_k[i] dw_l[i]."""
    A = [0] * 7
    for k in range(4):
        for l in range(4):
            if k + l < nsums:
                A[k + l] += int(np.dot(xd[:, k].astype(np.int64), wd[:, l].astype(np.int64)))
    return A


def value(A):
    return sum(a << (8 * (6 - g)) for g, a in enumerate(A))


def test_digit_split_reconstructs():
    rng = np.random.default_rng(0)
    lim = 1 << 30
    xs = list(rng.integers(-lim + 1, lim, 20000)) + [0, 1, -1, lim - 1, -lim + 1, 127, 128, -128, -129,
                                                     0x7F7F7F, -0x808080, 0x808080]
    for X in xs:
        d = digits(X)
        assert abs(d[0]) <= 64 and all(-128 <= v <= 127 for v in d[1:])
        assert d[0] * (1 << 24) + d[1] * (1 << 16) + d[2] * (1 << 8) + d[3] == X


@pytest.mark.parametrize("D", [8, 256, 2048])
def test_plane_products_exact_and_dropped_bound(D):
    rng = np.random.default_rng(D)
    lim = 1 << 30
    for trial in range(4):
        X = rng.integers(-lim + 1, lim, D)
        W = rng.integers(-lim + 1, lim, D)
        xd = np.array([digits(v) for v in X], dtype=np.int64)
        wd = np.array([digits(v) for v in W], dtype=np.int64)
        exact = sum(int(a) * int(b) for a, b in zip(X, W))
        A7 = plane_sums(xd, wd, 7)
        # every sum fits the int32 accumulators for D < 32768
        assert all(abs(a) < 4 * D * (1 << 14) for a in A7)
        assert value(A7) == exact
        A5 = plane_sums(xd, wd, 5)
        assert abs(exact - value(A5)) <= D * ((1 << 23) + (1 << 14))


def test_dropped_bound_is_tight():
    # every element's two lower digits at -128 (X = ...  0x808080 pattern)
    D = 64
    X = np.full(D, -0x808080, dtype=np.int64)
    xd = np.array([digits(v) for v in X], dtype=np.int64)
    assert list(xd[0]) == [0, -128, -128, -128]
    exact = sum(int(a) * int(a) for a in X)
    dropped = exact - value(plane_sums(xd, xd, 5))
    assert dropped == D * ((1 << 23) + (1 << 14))


# ---- the split-K finish's fp64 decision (logit_from_digit_sums<5>) ----
#
# The sum is known to lie within B 2^lsb of V 2^lsb (V the 13-product digit
# total, |V| < 2^80). The kernel converts V to fp64 as (V >> 32) 2^32 + the
# low 32 bits (one rounding), scales by 2^lsb, widens the interval by
# 2^-52 |s| (rounded up) and decides when both ends give the same bf16
# logit. The model below repeats those steps with Python floats (IEEE
# fp64, round-to-nearest) and directed roundings emulated exactly; the test
# checks that every decision equals the exact logit of every sum the
# interval allows.
import math
from fractions import Fraction


def _round_dir(a_plus_b: Fraction, t: float, up: bool) -> float:
    if up and Fraction(t) < a_plus_b:
        return math.nextafter(t, math.inf)
    if not up and Fraction(t) > a_plus_b:
        return math.nextafter(t, -math.inf)
    return t


def _add_dir(a: float, b: float, up: bool) -> float:
    return _round_dir(Fraction(a) + Fraction(b), a + b, up)


def _rn32(q: Fraction) -> np.float32:
    """Round-to-nearest-even of a rational to fp32 (normal range)."""
    if q == 0:
        return np.float32(0.0)
    sgn = -1 if q < 0 else 1
    a = abs(q)
    e = a.numerator.bit_length() - a.denominator.bit_length()
    if Fraction(2) ** e > a:
        e -= 1
    m = a / Fraction(2) ** (e - 23)  # in [2^23, 2^24)
    n, r = divmod(m.numerator, m.denominator)
    if 2 * r > m.denominator or (2 * r == m.denominator and n & 1):
        n += 1
    return np.float32(sgn * math.ldexp(n, e - 23))


def _bf16_bits(f: np.float32) -> int:
    u = int(np.float32(f).view(np.uint32))
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF


def _logit(f32: np.float32, bias: np.float32) -> int:
    return _bf16_bits(np.float32(f32) + bias)


def _fp64_decision(V: int, lsb: int, B: int, bias: np.float32):
    v = float(V >> 32) * 4294967296.0 + float(V & 0xFFFFFFFF)
    s = math.ldexp(v, lsb)
    err = _add_dir(math.ldexp(float(B), lsb), abs(s) * 2.0**-52, up=True)
    lo = _add_dir(s, -err, up=False)
    hi = _add_dir(s, err, up=True)
    a, b = _logit(np.float32(lo), bias), _logit(np.float32(hi), bias)
    return a == b, a


def test_fp64_decision_matches_exact_logit():
    rng = np.random.default_rng(7)
    D = 4096
    decided_n = 0
    cases = 0
    for trial in range(3000):
        lsb = int(rng.integers(-70, -50))
        B = D * ((1 << 23) + (1 << 14)) + int(rng.integers(0, 3)) * (1 << 30)
        bias = np.float32(0.0 if trial % 2 else rng.normal(0, 2))
        if trial % 3 == 0:
            V = int(rng.integers(-(1 << 62), 1 << 62)) * int(rng.integers(1, 1 << 16))
        else:
            # just beside a bf16 rounding boundary of the logit
            f = np.float32(rng.normal(0, 1.5))
            u = int(np.float32(f).view(np.uint32)) & 0xFFFF0000
            mid = np.uint32(u | 0x8000).view(np.float32)
            y = Fraction(float(mid)) - Fraction(float(bias))
            V = int(y / Fraction(2) ** lsb) + int(rng.integers(-4 * B, 4 * B))
        V = max(min(V, (1 << 80) - 1), -(1 << 80) + 1)
        ok, lb = _fp64_decision(V, lsb, B, bias)
        cases += 1
        if not ok:
            continue
        decided_n += 1
        for d in (-B, -B // 2, 0, B // 3, B):
            exact = _rn32(Fraction(V + d) * Fraction(2) ** lsb)
            assert _logit(exact, bias) == lb, (V, lsb, B, d, float(bias))
    # the boundary cases leave some undecided; the rest are decided
    assert 0.4 * cases < decided_n < cases
