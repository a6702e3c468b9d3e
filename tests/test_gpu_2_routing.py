"""GPU routing parity: the router (logits, probabilities, top-k indices and
weights) and the permutation are bit-exact with the oracle's routing contract."""
import numpy as np
import pytest
import torch

import oracle as O
from conftest import bf16_np
from mlxr_moe import synth
from mlxr_moe.moe import MoeConfig

pytestmark = pytest.mark.gpu


def _router_block(D, E, K, zipf=False, seed=0):
    """A block whose router is synthesised; experts are irrelevant here."""
    from mlxr_moe import ops
    from mlxr_moe.moe import Qwen35MoeBlock, QuantizedSwitchLinear, SplitSwitchFfn

    cfg = MoeConfig(D, E, K, 128, bits=4)
    router = ops.synth_normal_bf16(seed, synth.STREAM_ROUTER, (E, D), 0.02)
    dummy = QuantizedSwitchLinear.from_switch_linear(ops.synth_normal_bf16(seed, 1, (1, 128, D), 0.02), 64, 4)
    bias = synth.zipf_bias(E, D, seed) if zipf else None
    return Qwen35MoeBlock(cfg, router, SplitSwitchFfn(dummy, dummy, dummy), router_bias=bias)


@pytest.mark.parametrize(
    "D,E,K,T,zipf",
    [
        (2048, 128, 8, 32, False),    # C1
        (2048, 128, 8, 1, False),     # C2
        (2048, 128, 8, 64, False),    # C2
        (2048, 128, 8, 4096, True),   # C3 (Zipf-biased logits)
        (2048, 512, 10, 2048, False), # C4 router (subset of the 16384 tokens)
        (4096, 128, 8, 256, True),    # C5 decode batch
        (4096, 128, 8, 256, False),   # C5 decode sizes without a bias (small logits reach the fallback)
        (2048, 128, 8, 5, False),     # split router, 2 tokens per block
        (2048, 128, 8, 20, True),     # split router, 4 tokens per block, ragged last block
        (2176, 72, 6, 300, False),    # tiled router: partial token tile, partial expert tile, partial D block
        (2176, 72, 6, 17, False),     # split router with a partial expert group and D block
    ],
)
def test_router_bitexact(D, E, K, T, zipf):
    blk = _router_block(D, E, K, zipf)
    x = synth.make_input(T, D)
    idx, w, lg, pr = blk.router(x, want_logits=True)
    torch.cuda.synchronize()
    bias = None if blk.router_bias is None else blk.router_bias.cpu().numpy()
    oi, ow, olg, opr = O.router(bf16_np(x), bf16_np(blk.gate), K, bias, True, want_logits=True)
    np.testing.assert_array_equal(bf16_np(lg), olg)
    np.testing.assert_array_equal(bf16_np(pr), opr)
    np.testing.assert_array_equal(idx.cpu().numpy(), oi)
    np.testing.assert_array_equal(bf16_np(w), ow)


def test_router_ties_bitexact():
    """Duplicated router rows give equal probabilities; ties go to the lower expert."""
    blk = _router_block(2048, 128, 8)
    g = blk.gate.clone()
    g[5] = g[77]
    g[6] = g[77]
    g[100] = g[2]
    blk.gate.copy_(g)
    x = synth.make_input(512, 2048, stream_offset=3)
    idx, w = blk.router(x)
    oi, ow = O.router(bf16_np(x), bf16_np(blk.gate), 8)
    np.testing.assert_array_equal(idx.cpu().numpy(), oi)
    np.testing.assert_array_equal(bf16_np(w), ow)
    rows = idx.cpu().numpy()
    both = [(list(r).index(5), list(r).index(77)) for r in rows if 5 in r and 77 in r]
    assert both and all(a < b for a, b in both)


@pytest.mark.parametrize("T,K,E", [(1, 8, 128), (33, 8, 128), (4096, 8, 128), (16384, 10, 512)])
def test_permute_bitexact(T, K, E):
    D = 256
    blk = _router_block(D, E, K)
    x = synth.make_input(T, D, stream_offset=5)
    g = torch.Generator(device="cpu").manual_seed(T)
    # skewed indices: many rows on few experts, some experts empty
    idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).to(torch.int32)
    idx = torch.where(idx % 3 == 0, idx % 7, idx).to(torch.int32)
    idx_d = idx.cuda()
    counts, offsets, srt, inv, xs = blk.permute(idx_d, x)
    torch.cuda.synchronize()
    oc, oo, osrt, oinv = O.permute(idx.numpy(), E)
    np.testing.assert_array_equal(counts.cpu().numpy(), oc)
    np.testing.assert_array_equal(offsets.cpu().numpy(), oo)
    np.testing.assert_array_equal(srt.cpu().numpy(), osrt)
    np.testing.assert_array_equal(inv.cpu().numpy(), oinv)
    ref = x[(srt.long() // K)]
    assert torch.equal(xs, ref)


def test_permute_bad_index_reports_status():
    from mlxr_moe import MlxrError, _lib

    blk = _router_block(256, 16, 2)
    x = synth.make_input(8, 256)
    idx = torch.zeros((8, 2), dtype=torch.int32, device="cuda")
    idx[3, 1] = 9999
    blk.permute(idx, x)
    with pytest.raises(MlxrError) as ei:
        blk.status()
    assert ei.value.status == _lib.ERR_DEVICE_INDEX


@pytest.mark.parametrize("D,T", [(2048, 3), (2048, 100), (2048, 300), (2048, 1000), (32768, 3), (32768, 100)])
def test_router_undecided_and_non_finite_logits(D, T):
    """Logits the fast paths cannot decide go through the exact sum: a token
    whose sum with expert 5 is 1 + 2^-8 + 2^-24 + 2^-60 (the fp32 tie is broken
    only by the 2^-60 term, below fp64's reach and below the tensor-core
    path's digit range), and tokens holding inf or NaN. D = 2048 runs the
    int8 tensor-core router (split-K form for T <= 256, direct beyond);
    D = 32768 is past its int32 accumulator bound and runs the fp64 split
    (T = 3) and fused (T = 100) routers. All must equal the oracle's logits
    (NaN compared as NaN) and, for finite tokens, its routing."""
    E, K = 128, 8
    blk = _router_block(D, E, K)
    g = blk.gate.clone()
    g[5] = 0
    g[5, :4] = torch.tensor([1.0, 1.0, 1.0, 2.0**-30], dtype=torch.bfloat16)
    blk.gate.copy_(g)
    x = synth.make_input(T, D, stream_offset=11).clone()
    x[1] = 0
    x[1, :4] = torch.tensor([1.0, 2.0**-8, 2.0**-24, 2.0**-30], dtype=torch.bfloat16)
    x[2, 17] = float("inf")
    if T > 100:
        x[T - 1, 3] = float("nan")
        x[T // 2, 0] = float("-inf")
    idx, w, lg, pr = blk.router(x, want_logits=True)
    torch.cuda.synchronize()
    oi, ow, olg, opr = O.router(bf16_np(x), bf16_np(blk.gate), K, None, True, want_logits=True)
    got, want = bf16_np(lg), olg
    gnan = ((got & 0x7F80) == 0x7F80) & ((got & 0x7F) != 0)
    wnan = ((want & 0x7F80) == 0x7F80) & ((want & 0x7F) != 0)
    np.testing.assert_array_equal(gnan, wnan)
    np.testing.assert_array_equal(np.where(gnan, 0, got), np.where(wnan, 0, want))
    assert got[1, 5] == 0x3F81  # bf16(fp32(1 + 2^-8 + 2^-24 + 2^-60)) = 1 + 2^-7
    xf = bf16_np(x)
    finite = ((xf & 0x7F80) != 0x7F80).all(1)
    np.testing.assert_array_equal(idx.cpu().numpy()[finite], oi[finite])
    np.testing.assert_array_equal(bf16_np(w)[finite], ow[finite])
