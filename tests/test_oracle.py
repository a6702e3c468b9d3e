"""CPU tests of the oracle: the relations the reference's own tests assert,
the routing contract, and the committed golden fixtures."""
import os
import sys

import numpy as np
import pytest

import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_golden as G  # noqa: E402

FX = np.load(os.path.join(HERE, "golden", "moe_small.npz"))


def rng_normal(seed, stream, shape, scale=1.0):
    return O.bf16_to_f32(O.normal_bf16(seed, stream, shape, scale))


# ------------------------------------------- reference test relations ------
def test_quantize_dequantize_reference_bound():
    """crates/mlxr/src/ops/quantization.rs:299-315: shapes and max error <= 127/2^bits."""
    x = (np.ones((128, 1), np.float32) * np.arange(512, dtype=np.float32)[None, :]).astype(np.float32)
    for bits in (2, 4, 8):
        el_per_int = 32 // bits
        q, s, b = O.quantize(x, 128, bits)
        assert q.shape == (128, 512 // el_per_int)
        assert s.shape == (128, 4) and b.shape == (128, 4)
        xh = O.dequantize(q, s, b, 128, bits)
        assert np.abs(x - xh).max() <= 127.0 / (1 << bits)


def mlx_affine_quantize_np(w32, gs, bits):
    """Independent numpy restatement of MLX's affine quantiser (ml-explore/mlx
    v0.31.2 `affine_quantize`, mlx/ops.cpp, CPU kernel in
    mlx/backend/cpu/quantized.cpp), every step an IEEE fp32 operation:
    returns codes [rows, cols] and the fp32 (scale, bias) per group."""
    f = np.float32
    rows, cols = w32.shape
    g = w32.reshape(rows, cols // gs, gs).astype(f)
    mn, mx = g.min(-1), g.max(-1)
    nbins = f((1 << bits) - 1)
    min_edge = np.abs(mn) > np.abs(mx)
    sc = np.maximum((mx - mn) / nbins, f(1e-7)).astype(f)
    sc = np.where(min_edge, sc, -sc).astype(f)
    edge = np.where(min_edge, mn, mx).astype(f)
    q0 = np.rint(edge / sc).astype(f)
    nz = q0 != 0
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(nz, edge / np.where(nz, q0, f(1)), sc).astype(f)
    bi = np.where(nz, edge, f(0)).astype(f)
    q = np.clip(np.rint((g - bi[..., None]) / sc[..., None]), 0, nbins).astype(np.uint32)
    return q.reshape(rows, cols), sc, bi, q0


def pack_codes(q, bits):
    per = 32 // bits
    r, c = q.shape
    q = q.reshape(r, c // per, per).astype(np.uint64)
    sh = (np.arange(per, dtype=np.uint64) * bits)[None, None, :]
    return (q << sh).sum(-1).astype(np.uint32)


@pytest.mark.parametrize("bits", [2, 4, 8])
@pytest.mark.parametrize("gs", [32, 64, 128])
def test_quantize_is_mlx_affine_quantize(bits, gs):
    """The oracle's bytes equal an independent restatement of MLX's
    affine_quantize on random bf16 groups plus edge groups (all zero,
    constant, one-signed, spanning zero, |min| == |max|)."""
    w = O.normal_bf16(0, 150 + bits, (64, 512), 0.02)
    wf = O.bf16_to_f32(w).copy()
    wf[0, :gs] = 0.0                                  # all zero: q0 == 0, bias 0
    wf[1, :gs] = 0.03125                              # constant positive
    wf[2, :gs] = -np.abs(wf[2, :gs])                  # all non-positive
    wf[3, :gs] = np.abs(wf[3, :gs])                   # all non-negative
    wf[4, :gs] = np.linspace(-0.5, 0.5, gs)           # |min| == |max|
    wf[5, :gs] = np.linspace(-1.0, 0.875, gs)
    wf[5, 1] = 0.0                                    # spans zero, holds a 0
    wb = O.f32_to_bf16(wf.astype(np.float32))
    q, s, b = O.quantize(wb, gs, bits)
    rq, rs, rb, _ = mlx_affine_quantize_np(O.bf16_to_f32(wb), gs, bits)
    np.testing.assert_array_equal(q, pack_codes(rq, bits))
    np.testing.assert_array_equal(s, O.f32_to_bf16(rs))
    np.testing.assert_array_equal(b, O.f32_to_bf16(rb))
    # float32 input: the pair is stored unrounded
    q32, s32, b32 = O.quantize(O.bf16_to_f32(wb).astype(np.float32), gs, bits)
    np.testing.assert_array_equal(q32, pack_codes(rq, bits))
    np.testing.assert_array_equal(s32, rs)
    np.testing.assert_array_equal(b32, rb)


def test_quantize_mlx_hand_computed_groups():
    """Groups worked by hand (4-bit, group 8, float32 in and out)."""
    w = np.array([
        [-1.0, 0.0, 0.125, 0.25, 0.5, 0.625, 0.75, 0.875],   # |min| > |max|
        [-0.5, -0.25, 0.0, 0.25, 0.5, 1.0, 1.25, 1.5],       # |max| > |min|
        [0.0] * 8,                                           # all zero
    ], np.float32)
    w32 = np.tile(w, (1, 4))  # group size 32 (the smallest the ABI takes): 4 copies
    q, s, b = O.quantize(w32, 32, 4)
    codes = ((q[:, :, None] >> (np.arange(8, dtype=np.uint32) * 4)) & 15).reshape(3, 32)[:, :8]
    # Row 0: scale = (0.875 + 1) / 15 = 0.125 > 0, edge = min = -1, q0 = -8,
    # scale = -1 / -8 = 0.125, bias = -1; codes (w + 1) / 0.125; 0 -> 8 -> 0.0.
    assert s[0, 0] == np.float32(0.125) and b[0, 0] == np.float32(-1.0)
    np.testing.assert_array_equal(codes[0], [0, 8, 9, 10, 12, 13, 14, 15])
    # Row 1: |max| >= |min| -> scale = -(2 / 15), edge = max = 1.5,
    # q0 = rint(1.5 / -0.1333) = rint(-11.25) = -11, scale = 1.5 / -11 < 0,
    # bias = 1.5; the code of 0 is rint(-1.5 / scale) = 11.
    assert s[1, 0] == np.float32(1.5) / np.float32(-11.0) and b[1, 0] == np.float32(1.5)
    assert codes[1, 2] == 11 and codes[1, 7] == 0
    # Row 2: scale = -max(0, 1e-7) = -1e-7, q0 = 0 -> bias 0, codes 0.
    assert s[2, 0] == -np.float32(1e-7) and b[2, 0] == 0.0
    assert (codes[2] == 0).all()
    # The code of 0 dequantises to 0 within the fp32 rounding of scale * q0.
    for r, c0 in ((0, 8), (1, 11)):
        assert abs(np.float32(s[r, 0]) * np.float32(c0) + b[r, 0]) <= 4 * np.finfo(np.float32).eps


def test_quantize_mlx_properties_random():
    """On N(0, 0.02) bf16 groups: the scale is negative exactly when
    |max| >= |min|, the bias is the edge, and the element 0 dequantises to
    within the bf16 rounding of the scale times |q0| of zero."""
    w = O.normal_bf16(0, 160, (256, 1024), 0.02)
    wf = O.bf16_to_f32(w).copy()
    wf[:, ::64] = 0.0  # every group holds a 0
    wb = O.f32_to_bf16(wf.astype(np.float32))
    q, s, b = O.quantize(wb, 64, 4)
    g = O.bf16_to_f32(wb).reshape(256, 16, 64)
    mn, mx = g.min(-1), g.max(-1)
    sf, bf = O.bf16_to_f32(s), O.bf16_to_f32(b)
    assert ((sf < 0) == (np.abs(mx) >= np.abs(mn))).all()
    edge = np.where(np.abs(mn) > np.abs(mx), mn, mx)
    np.testing.assert_array_equal(bf, edge)
    wh = O.dequantize(q, s, b, 64, 4).reshape(256, 16, 64)[..., 0]
    _, rs, _, q0 = mlx_affine_quantize_np(O.bf16_to_f32(wb), 64, 4)
    assert (np.abs(wh) <= np.abs(q0) * np.abs(rs) * 2.0**-8 + 1e-12).all()


def test_quantized_matmul_reference_relation():
    """quantization.rs:318-341: qmm(x, w) == x @ dequant(w) within 1e-3 (transpose=false)."""
    m, n, k = 32, 128, 128
    x = rng_normal(0, 100, (m, k)) / np.sqrt(k)
    w = rng_normal(0, 101, (k, n)) / np.sqrt(k)
    wq, s, b = O.quantize(w.astype(np.float32), 64, 4)
    wh = O.dequantize(wq, s, b, 64, 4)
    yq = O.quantized_matmul(x.astype(np.float32), wq, s, b, transpose=False, group_size=64, bits=4)
    yh = x.astype(np.float64) @ wh.astype(np.float64)
    assert yq.shape == yh.shape
    assert np.abs(yq - yh).max() < 1e-3


def test_gather_qmm_reference_relation():
    """quantization.rs:344-421: gather_qmm == gather_mm on dequantised transposed weights (1e-4)."""
    m, n, k = 32, 64, 64
    w = rng_normal(0, 102, (3, n, k)).astype(np.float32)
    wq, s, b = O.quantize(w, 64, 4)
    w_hat = np.swapaxes(O.dequantize(wq, s, b, 64, 4), -1, -2)
    rhs = np.array([2, 1], np.int32)
    for x_batch, lhs in ((1, np.array([0, 0], np.int32)), (5, np.array([0, 2], np.int32))):
        x = rng_normal(0, 103 + x_batch, (x_batch, m, k)).astype(np.float32)
        c1 = O.gather_mm(x, w_hat, lhs, rhs)
        c2 = O.gather_qmm(x, wq, s, b, lhs, rhs, True, 64, 4)
        np.testing.assert_allclose(c2, c1, rtol=1e-4, atol=1e-4)


def test_gather_mm_reference_cases():
    """arithmetic.rs:3099-3196: gather_mm == take + matmul, incl. the sorted-rhs case."""
    a = rng_normal(0, 110, (1, 32, 32)).astype(np.float32)
    b = rng_normal(0, 111, (3, 32, 32)).astype(np.float32)
    rhs = np.array([2, 1], np.int32)
    ref = np.stack([a[0] @ b[2], a[0] @ b[1]])
    np.testing.assert_allclose(O.gather_mm(a, b, np.array([0, 0], np.int32), rhs), ref, rtol=1e-5, atol=1e-5)
    a5 = rng_normal(0, 112, (5, 32, 32)).astype(np.float32)
    ref = np.stack([a5[0] @ b[2], a5[2] @ b[1]])
    np.testing.assert_allclose(O.gather_mm(a5, b, np.array([0, 2], np.int32), rhs), ref, rtol=1e-5, atol=1e-5)
    a100 = rng_normal(0, 113, (100, 1, 100)).astype(np.float32)
    b8 = rng_normal(0, 114, (8, 100, 100)).astype(np.float32)
    r = np.sort(O.normal_bf16(0, 115, (100,), 1.0).view(np.int16).astype(np.int64) % 8).astype(np.int32)
    ref = np.stack([a100[i] @ b8[r[i]] for i in range(100)])
    np.testing.assert_allclose(O.gather_mm(a100, b8, np.arange(100, dtype=np.int32), r), ref, rtol=1e-4, atol=1e-4)


def test_swiglu_matches_manual_silu_multiply():
    """activations.rs:341-351 on the reference's own values."""
    gate = np.array([1.0, -1.0, 0.5, 2.0], np.float32)
    x = np.array([1.0, 2.0, 3.0, 4.0], np.float32)
    fused = gate / (1 + np.exp(-gate)) * x
    manual = gate * (1 / (1 + np.exp(-gate))) * x
    assert np.abs(fused - manual).max() < 1e-5


# --------------------------------------------------- routing contract ------
def test_exp_route_accuracy_and_monotone():
    t = np.linspace(-80.0, 0.0, 200001, dtype=np.float32)
    e = O.exp_route(t).astype(np.float64)
    ex = np.exp(t.astype(np.float64))
    assert (np.abs(e - ex) / ex).max() < 2.5 * 2.0**-24
    assert (np.diff(e) >= 0).all()
    assert O.exp_route(np.array([0.0], np.float32))[0] == 1.0
    assert O.exp_route(np.array([-200.0], np.float32))[0] == 0.0
    # subnormal results are produced with a single rounding
    sub = O.exp_route(np.array([-100.0], np.float32))[0]
    assert 0.0 < sub < 1.2e-38


def test_router_topk_order_and_ties():
    D, E, K, T = 256, 32, 4, 64
    x = O.normal_bf16(0, 120, (T, D), 1.0)
    wg = O.normal_bf16(0, 121, (E, D), 0.02)
    wg[7] = wg[3]  # duplicated rows -> identical logits -> tie broken by lower index
    wg[20] = wg[3]
    idx, w, lg, pr = O.router(x, wg, K, want_logits=True)
    p = O.bf16_to_f32(pr)
    for t in range(T):
        key = sorted(range(E), key=lambda e: (-p[t, e], e))[:K]
        assert list(idx[t]) == key
        assert len(set(idx[t])) == K
    sel = (idx == 3).any(1)
    assert sel.any()
    for t in np.nonzero(sel)[0]:
        row = list(idx[t])
        if 7 in row:
            assert row.index(3) < row.index(7)
    ws = O.bf16_to_f32(w).sum(1)
    assert np.abs(ws - 1).max() < 0.02


def test_permute_is_stable_counting_sort():
    T, K, E = 300, 8, 64
    idx = (O.normal_bf16(0, 130, (T, K), 1.0).view(np.int16).astype(np.int64) % E).astype(np.int32)
    counts, offsets, srt, inv = O.permute(idx, E)
    flat = idx.reshape(-1)
    np.testing.assert_array_equal(srt, np.argsort(flat, kind="stable"))
    np.testing.assert_array_equal(inv[srt], np.arange(T * K))
    np.testing.assert_array_equal(counts, np.bincount(flat, minlength=E))
    np.testing.assert_array_equal(offsets, np.concatenate([[0], np.cumsum(counts)]))


# ------------------------------------------------------ golden fixtures ----
@pytest.mark.parametrize("name", list(G.BLOCKS))
def test_golden_block(name):
    cfg, W, x = G.small_block(**G.BLOCKS[name])
    for k, v in G.flat(f"{name}/", W).items():
        assert G.digest(v) == str(FX[k + ".sha256"]), f"generator/quantiser drifted for {k}"
    np.testing.assert_array_equal(x, FX[f"{name}/x"])
    o_st, idx, w = O.moe_block(cfg, W, x, "staged")
    o_fu, idx2, w2 = O.moe_block(cfg, W, x, "fused")
    np.testing.assert_array_equal(idx, FX[f"{name}/idx"])
    np.testing.assert_array_equal(idx2, FX[f"{name}/idx"])
    np.testing.assert_array_equal(w, FX[f"{name}/w"])
    np.testing.assert_array_equal(o_st, FX[f"{name}/out_staged"])
    np.testing.assert_array_equal(o_fu, FX[f"{name}/out_fused"])
    # staged vs fused stay within the block tolerance
    d = np.abs(O.bf16_to_f32(o_st).astype(np.float64) - O.bf16_to_f32(o_fu))
    assert (d <= 2e-2 + 1e-2 * np.abs(O.bf16_to_f32(o_st))).all()


def test_golden_quantiser_and_generator():
    x = (np.ones((128, 1), np.float32) * np.arange(512, dtype=np.float32)[None, :]).astype(np.float32)
    for b in (2, 4, 8):
        q, s, bb = O.quantize(x, 128, b)
        np.testing.assert_array_equal(q, FX[f"quant_arange/b{b}.weight"])
        np.testing.assert_array_equal(s, FX[f"quant_arange/b{b}.scales"])
        np.testing.assert_array_equal(bb, FX[f"quant_arange/b{b}.biases"])
    for st in (0, 1, 8):
        np.testing.assert_array_equal(O.normal_bf16(0, st, (4096,), 1.0), FX[f"normal/seed0_stream{st}"])
    z = O.bf16_to_f32(O.normal_bf16(0, 8, (1 << 16,), 1.0))
    assert abs(z.mean()) < 0.02 and abs(z.std() - 1) < 0.02


def test_block_empty_and_single_token():
    cfg, W, x = G.small_block(seed=3, D=256, E=16, K=4, I=128, T=1, bits=4)
    o, idx, w = O.moe_block(cfg, W, x, "fused")
    assert o.shape == (1, 256) and idx.shape == (1, 4)
    o0, idx0, _ = O.moe_block(cfg, W, x[:0], "fused")
    assert o0.shape == (0, 256) and idx0.shape == (0, 4)


# ------------------------------------------- exact router dot product ----
def _bf16_value(b):
    """Exact value of bf16 bits as a Fraction (finite only)."""
    from fractions import Fraction

    be, f = (int(b) >> 7) & 0xFF, int(b) & 0x7F
    m = (f | 0x80) if be else f
    p = (be if be else 1) - 134
    v = Fraction(m) * (Fraction(2) ** p)
    return -v if int(b) & 0x8000 else v


def _rn32(F):
    """Fraction -> fp32 bits, round to nearest, ties to even (exact zero +0)."""
    from fractions import Fraction

    if F == 0:
        return 0
    sign = 0x80000000 if F < 0 else 0
    a = abs(F)
    e = a.numerator.bit_length() - a.denominator.bit_length()
    if Fraction(2) ** e > a:
        e -= 1
    if e > 127:
        return sign | 0x7F800000
    q = max(e - 23, -149)
    s = a / (Fraction(2) ** q)
    mant = int(s)
    rem = s - mant
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and mant & 1):
        mant += 1
    if mant == 1 << 24:
        mant >>= 1
        q += 1
    if mant >= 1 << 23:
        if q + 23 > 127:
            return sign | 0x7F800000
        return sign | ((q + 150) << 23) | (mant & 0x7FFFFF)
    return sign | mant


def _f32_bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def test_dot_rn32_matches_exact_rational_sum():
    """The logit's sum: the exact dot product rounded once to fp32, checked
    against rational arithmetic on vectors with wide exponent ranges,
    subnormals, cancellation and ties."""
    rng = np.random.default_rng(7)
    rows, D = 48, 72
    x = np.empty((rows, D), np.uint16)
    w = np.empty((rows, D), np.uint16)
    for r in range(rows):
        # random sign, exponent field in a row-specific window, random mantissa
        lo = int(rng.integers(0, 200))
        hi = min(254, lo + int(rng.integers(1, 60)))
        for arr in (x, w):
            ex = rng.integers(lo, hi + 1, D)
            arr[r] = (rng.integers(0, 2, D) << 15) | (ex << 7) | rng.integers(0, 128, D)
    # exact cancellation: the second half negates the first
    x[0, D // 2:] = x[0, :D // 2] ^ 0x8000
    w[0, D // 2:] = w[0, :D // 2]
    # a fp32 tie that only the tiny term breaks: 1 + 2^-8 + 2^-24 + 2^-60
    x[1] = 0
    w[1] = 0
    x[1, :4] = [0x3F80, 0x3B80, 0x3380, 0x3080]  # 1, 2^-8, 2^-24, 2^-30
    w[1, :4] = [0x3F80, 0x3F80, 0x3F80, 0x3080]  # 1, 1, 1, 2^-30
    # the same without the tiny term: a tie, rounds to even
    x[2] = x[1]
    w[2] = w[1]
    x[2, 3] = 0
    # all zero, and products that cancel to exactly zero
    x[3] = 0
    x[4, :] = 0
    x[4, :2] = [0x3F80, 0xBF80]
    w[4, :] = 0
    w[4, :2] = [0x4000, 0x4000]
    got = _f32_bits(O.dot_rn32(x, w))
    for r in range(rows):
        F = sum(_bf16_value(a) * _bf16_value(b) for a, b in zip(x[r], w[r]))
        assert got[r] == _rn32(F), (r, hex(got[r]), hex(_rn32(F)))
    assert got[1] == 0x3F808001  # 1 + 2^-8 + 2^-23: the 2^-60 term decides the tie
    assert got[2] == 0x3F808000
    assert got[3] == 0 and got[4] == 0  # exact zeros are +0


def test_dot_rn32_non_finite_operands():
    one, inf, ninf, nan, zero = 0x3F80, 0x7F80, 0xFF80, 0x7FC0, 0x0000
    cases = [
        ([inf, one], [one, one], 0x7F800000),
        ([inf, ninf], [one, ninf], 0x7F800000),   # +inf and (-inf * -inf) = +inf
        ([inf, ninf], [one, one], None),          # +inf + -inf -> NaN
        ([inf, one], [zero, one], None),          # inf * 0 -> NaN
        ([nan, one], [one, one], None),
        ([ninf, one], [one, one], 0xFF800000),
    ]
    for xs, ws, want in cases:
        got = _f32_bits(O.dot_rn32(np.array([xs], np.uint16), np.array([ws], np.uint16)))[0]
        if want is None:
            assert (got & 0x7F800000) == 0x7F800000 and (got & 0x7FFFFF) != 0
        else:
            assert got == want


def test_router_logits_are_rounded_exact_sums():
    """route_logit = bf16(fp32(exact sum) + bias) on the router's own shapes."""
    D, E, T = 512, 16, 8
    x = O.normal_bf16(0, 140, (T, D), 1.0)
    wg = O.normal_bf16(0, 141, (E, D), 0.02)
    bias = np.linspace(-1.0, 1.0, E).astype(np.float32)
    _, _, lg, _ = O.router(x, wg, 4, bias, True, want_logits=True)
    s = O.dot_rn32(np.repeat(x, E, 0), np.tile(wg, (T, 1))).reshape(T, E)
    want = O.f32_to_bf16((s + bias[None, :]).astype(np.float32))
    np.testing.assert_array_equal(lg, want)
