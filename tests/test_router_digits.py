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
