"""CPU tests of the oracle's Gemma 4 MoE branch (gemma4/text/text.rs:622-664,
activations.rs:309-331, nn/switch.rs:242-345): the router's relations as the
reference's own test asserts them (router_post_matches_manual,
activations.rs:378-398), GeGLU against a manual gelu_approx(gate) * up, and
the whole branch against an independent float64 restatement."""
import numpy as np
import pytest

import oracle as O

D, E, K, I = 256, 16, 4, 128
EPS = 1e-6


def bf(a):
    return O.bf16_to_f32(O.f32_to_bf16(np.asarray(a, np.float32)))


def weights(seed=0):
    g = lambda st, shape, sd: O.normal_bf16(seed, st, shape, sd)  # noqa: E731
    w = {
        "router": g(0, (E, D), 0.05),
        "router_norm": O.f32_to_bf16(np.float32(D ** -0.5) * (1.0 + O.bf16_to_f32(g(1, (D,), 0.1)))),
        "expert_scale": O.f32_to_bf16(1.0 + O.bf16_to_f32(g(2, (E,), 0.2))),
        "experts_norm": O.f32_to_bf16(1.0 + O.bf16_to_f32(g(3, (D,), 0.1))),
    }
    # bf16 inputs: the quantiser stores scales and biases in the weight dtype
    w["gate_up"] = O.quantize(g(4, (E, 2 * I, D), 0.02), 64, 4)
    w["down"] = O.quantize(g(5, (E, D, I), 0.02), 64, 4)
    return w


CFG = dict(hidden=D, num_experts=E, top_k=K, moe_intermediate=I, group_size=64, bits=4, eps=EPS)


def gelu_tanh(g):
    return 0.5 * g * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (g + 0.044715 * g ** 3)))


def manual_branch(w, x):
    """float64 restatement: rms_norm, scores, top-k, router_post, packed
    gate_up split, GeGLU, down, weighted sum."""
    xf = O.bf16_to_f32(x).astype(np.float64)
    inv = 1.0 / np.sqrt((xf ** 2).mean(axis=1, keepdims=True) + EPS)
    xr = bf(xf * inv * O.bf16_to_f32(w["router_norm"]))
    xe = bf(xf * inv * O.bf16_to_f32(w["experts_norm"]))
    scores = bf(xr.astype(np.float64) @ O.bf16_to_f32(w["router"]).astype(np.float64).T)
    idx = np.argsort(-scores, axis=1, kind="stable")[:, :K]
    top = np.take_along_axis(scores, idx, 1).astype(np.float64)
    p = np.exp(top - top[:, :1])
    p = bf(p / p.sum(axis=1, keepdims=True))
    wk = bf(p * O.bf16_to_f32(w["expert_scale"])[idx])
    gu = bf(O.dequantize(*w["gate_up"], 64, 4)).astype(np.float64)  # [E, 2I, D]
    dn = bf(O.dequantize(*w["down"], 64, 4)).astype(np.float64)     # [E, D, I]
    out = np.zeros_like(xf)
    for t in range(x.shape[0]):
        for k in range(K):
            e = idx[t, k]
            a = gu[e] @ xe[t]
            h = bf(gelu_tanh(a[:I]) * a[I:])
            y = bf(dn[e] @ h)
            out[t] += wk[t, k] * y
    return bf(out), idx, wk, scores


def test_router_post_matches_manual():
    """activations.rs:378-398: softmax over the picked scores times the
    picked per-expert scales, on the same example (scores 1..4, experts
    (1, 3) picked, scales 10..40), through the contract's exp and bf16 steps."""
    picked = np.array([2.0, 4.0], np.float32)
    scale = np.array([20.0, 40.0], np.float32)
    p = np.exp(picked - picked.max())
    manual = p / p.sum() * scale
    # The contract orders the picks by score: expert 3 first, then expert 1.
    ex = O.exp_route(np.array([0.0, 2.0 - 4.0], np.float32))
    got = bf(bf(ex / ex.sum(dtype=np.float32)) * scale[::-1])
    np.testing.assert_allclose(got, manual[::-1], rtol=1e-2)


def test_routing_matches_manual_and_is_deterministic():
    w = weights()
    x = O.normal_bf16(0, 10, (64, D), 1.0)
    _, idx, wk = O.gemma4_block(CFG, w, x, routing_only=True)
    _, idx2, wk2 = O.gemma4_block(CFG, w, x, routing_only=True)
    np.testing.assert_array_equal(idx, idx2)
    np.testing.assert_array_equal(wk, wk2)
    _, midx, mwk, scores = manual_branch(w, x)
    # Every picked expert's score is >= every unpicked one (ties broken by index).
    for t in range(x.shape[0]):
        picked = scores[t, idx[t]]
        rest = np.delete(scores[t], idx[t])
        assert picked.min() >= rest.max() - 1e-6
        assert np.all(np.diff(picked) <= 0)
    agree = (np.sort(idx, 1) == np.sort(midx, 1)).all(1).mean()
    assert agree >= 0.95, agree
    ok = (idx == midx).all(1)
    np.testing.assert_allclose(O.bf16_to_f32(wk)[ok], mwk[ok], rtol=2e-2, atol=1e-3)


def test_geglu_matches_manual_gelu_multiply():
    """GegluActivation (switch.rs:195-206): gelu_approx(gate) * up on the
    reference test's values, against the exp form the kernel evaluates."""
    g = np.array([1.0, -1.0, 0.5, 2.0], np.float64)
    u = np.array([1.0, 2.0, 3.0, 4.0], np.float64)
    manual = gelu_tanh(g) * u
    # 0.5 g (1 + tanh(y)) == g / (1 + exp(-2y)): the form the kernel uses.
    y = np.sqrt(2.0 / np.pi) * (g + 0.044715 * g ** 3)
    np.testing.assert_allclose(g / (1.0 + np.exp(-2.0 * y)) * u, manual, rtol=1e-12)


@pytest.mark.parametrize("T", [1, 7, 33])
def test_branch_matches_float64_restatement(T):
    w = weights(1)
    x = O.normal_bf16(1, 20 + T, (T, D), 1.0)
    out, idx, wk = O.gemma4_block(CFG, w, x)
    mout, midx, _, _ = manual_branch(w, x)
    ok = (idx == midx).all(1)
    assert ok.mean() >= 0.9
    np.testing.assert_allclose(O.bf16_to_f32(out)[ok], mout[ok], atol=2e-2, rtol=1e-2)


def test_empty_batch():
    w = weights()
    out, idx, wk = O.gemma4_block(CFG, w, np.zeros((0, D), np.uint16))
    assert out.shape == (0, D) and idx.shape == (0, K)


def test_golden_gemma4_branch():
    """The committed fixture (tests/golden/make_golden.py, `gemma4_small.npz`):
    the generator, the quantiser and the branch's routing and outputs are
    unchanged."""
    import os
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(here, "golden"))
    import make_golden as G

    fx = np.load(os.path.join(here, "golden", "gemma4_small.npz"))
    for name, args in G.GEMMA4.items():
        cfg, W, x = G.small_gemma4(**args)
        for k, v in G.flat(f"{name}/", W).items():
            assert G.digest(v) == str(fx[k + ".sha256"]), f"generator/quantiser drifted for {k}"
        np.testing.assert_array_equal(x, fx[f"{name}/x"])
        out, idx, w = O.gemma4_block(cfg, W, x)
        np.testing.assert_array_equal(idx, fx[f"{name}/idx"])
        np.testing.assert_array_equal(w, fx[f"{name}/w"])
        np.testing.assert_array_equal(out, fx[f"{name}/out"])
