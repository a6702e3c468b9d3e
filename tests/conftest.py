"""Shared test setup: import paths, the `gpu` marker, oracle/GPU helpers."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "oracle"), os.path.join(ROOT, "mlx-rs_b200"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


# Tolerance of the block outputs against the oracle (north star: bf16 outputs
# within max-abs 2e-2 and rtol 1e-2 with fp32 accumulation).
ATOL = 2e-2
RTOL = 1e-2


def bf16_np(t):
    """torch bf16 tensor -> numpy uint16 bit patterns (host)."""
    import torch

    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def np_bf16_to_torch(a, device="cuda"):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(device)


def to_f32(a_u16):
    return (a_u16.astype(np.uint32) << 16).view(np.float32)


def assert_mostly_tight(got_u16, want_u16, atol, rtol, max_frac, what="output"):
    """At most max_frac of the elements may fall outside the tight bound
    (bf16 outputs flip by an ulp or two when two fp32 accumulation orders
    straddle a rounding boundary)."""
    g = to_f32(got_u16).astype(np.float64)
    w = to_f32(want_u16).astype(np.float64)
    err = np.abs(g - w)
    frac = float((err > atol + rtol * np.abs(w)).mean())
    assert frac <= max_frac, f"{what}: {frac:.2e} of elements outside atol={atol} rtol={rtol} (allowed {max_frac})"
    return frac


def assert_close_bf16(got_u16, want_u16, atol=ATOL, rtol=RTOL, what="output"):
    g = to_f32(got_u16).astype(np.float64)
    w = to_f32(want_u16).astype(np.float64)
    assert np.isfinite(g).all(), f"{what}: non-finite values"
    err = np.abs(g - w)
    bad = err > atol + rtol * np.abs(w)
    assert not bad.any(), (
        f"{what}: {bad.sum()} of {bad.size} outside atol={atol} rtol={rtol}; max abs err {err.max():.3e}"
    )
    return float(err.max())
