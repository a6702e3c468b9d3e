"""The synthetic routing skew of the Zipf configurations (C3, C5).

The benchmark biases router logits by -beta * sigma * 1.1 * ln(rank) so that the
assignment histogram approximates Zipf(1.1) under the top-K-without-replacement
cap. These CPU tests route seeded C3/C5-shaped tokens through the oracle router
and check that the committed beta is the best fit among its neighbours and that
the skew does not depend on the hidden size.
"""
import numpy as np
import pytest

import oracle as O
from mlxr_moe import synth


def _ranks(E, seed=0):
    """synth.expert_ranks restated on the oracle's generator (same Philox stream)."""
    keys = O.normal_bf16(seed, synth.STREAM_RANK, (E,), 1.0)
    kf = (keys.astype(np.uint32) << 16).view(np.float32)
    order = np.argsort(kf, kind="stable")
    ranks = np.empty(E, np.int64)
    ranks[order] = np.arange(1, E + 1)
    return ranks


def _capped_zipf(E, K, s=synth.ZIPF_S):
    p = np.arange(1, E + 1, dtype=np.float64) ** -s
    p /= p.sum()
    cap = 1.0 / K
    while (p > cap + 1e-15).any():
        over = p > cap
        excess = (p[over] - cap).sum()
        p[over] = cap
        free = p < cap
        p[free] += excess * p[free] / p[free].sum()
    return p


def _shares(D, E, K, T, beta):
    wg = O.normal_bf16(0, synth.STREAM_ROUTER, (E, D), 0.02)
    x = O.normal_bf16(0, synth.STREAM_X + 16 * 7, (T, D), 1.0)
    r = _ranks(E)
    bias = (-beta * synth.router_logit_sigma(D) * synth.ZIPF_S * np.log(r.astype(np.float64))).astype(np.float32)
    idx, _ = O.router(x, wg, K, bias)
    cnt = np.bincount(idx.ravel(), minlength=E).astype(np.float64)
    share = np.zeros(E)
    share[r - 1] = cnt / cnt.sum()
    return share


def test_capped_target_is_a_distribution():
    p = _capped_zipf(128, 8)
    assert abs(p.sum() - 1.0) < 1e-12
    assert p.max() <= 1.0 / 8 + 1e-12
    assert np.all(np.diff(p) <= 1e-15)


@pytest.mark.parametrize("D,T", [(2048, 1024), (4096, 512)])
def test_committed_beta_is_the_local_best_fit(D, T):
    E, K = 128, 8
    p = _capped_zipf(E, K)
    l1 = {b: np.abs(_shares(D, E, K, T, b) - p).sum()
          for b in (synth.ZIPF_BETA - 0.12, synth.ZIPF_BETA, synth.ZIPF_BETA + 0.12)}
    assert l1[synth.ZIPF_BETA] < min(l1[synth.ZIPF_BETA - 0.12], l1[synth.ZIPF_BETA + 0.12]), l1
    top1 = _shares(D, E, K, T, synth.ZIPF_BETA)[0]
    assert 0.08 < top1 <= 1.0 / K + 1e-12


def test_skew_is_independent_of_hidden_size():
    a = _shares(2048, 128, 8, 1024, synth.ZIPF_BETA)
    b = _shares(4096, 128, 8, 1024, synth.ZIPF_BETA)
    assert abs(a[:8].sum() - b[:8].sum()) < 0.03
    assert abs(a[64:].sum() - b[64:].sum()) < 0.03
