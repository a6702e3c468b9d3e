"""GPU parity of the op family (quantize, dequantize, quantized_matmul,
gather_qmm, gather_mm) and the seeded generator, through the C ABI."""
import numpy as np
import pytest
import torch

import oracle as O
from conftest import bf16_np, np_bf16_to_torch, to_f32
from gpu_helpers import u32

pytestmark = pytest.mark.gpu


def test_synth_generator_matches_oracle():
    from mlxr_moe import ops

    for stream, n, sd in ((8, 1 << 20, 1.0), (1, 333_333, 0.02)):
        g = bf16_np(ops.synth_normal_bf16(0, stream, (n,), sd))
        o = O.normal_bf16(0, stream, (n,), sd)
        mism = int((g != o).sum())
        # fp64 log/cos/sin of CUDA and the host libm may differ in the last fp64
        # bit; after rounding to bf16 that shows up (if at all) as rare 1-ulp flips.
        assert mism <= 2, f"{mism} of {n} samples differ"


@pytest.mark.parametrize("bits,gs", [(4, 64), (8, 64), (2, 64), (4, 32), (4, 128)])
def test_quantize_bitexact_bf16(bits, gs):
    from mlxr_moe import ops

    w = ops.synth_normal_bf16(0, 40 + bits, (96, 1024), 0.02)
    wq, s, b = ops.quantize(w, gs, bits)
    oq, os_, ob = O.quantize(bf16_np(w), gs, bits)
    np.testing.assert_array_equal(u32(wq), oq)
    np.testing.assert_array_equal(bf16_np(s), os_)
    np.testing.assert_array_equal(bf16_np(b), ob)


def test_quantize_dequantize_reference_case_f32():
    """quantization.rs:299-315 on the GPU, f32 input, bit-exact with the oracle."""
    from mlxr_moe import ops

    x = torch.arange(512, dtype=torch.float32, device="cuda").expand(128, 512).contiguous()
    for bits in (2, 4, 8):
        wq, s, b = ops.quantize(x, 128, bits)
        assert tuple(wq.shape) == (128, 512 * bits // 32) and tuple(s.shape) == (128, 4)
        oq, os_, ob = O.quantize(x.cpu().numpy(), 128, bits)
        np.testing.assert_array_equal(u32(wq), oq)
        np.testing.assert_array_equal(s.cpu().numpy(), os_)
        xh = ops.dequantize(wq, s, b, 128, bits)
        np.testing.assert_array_equal(xh.cpu().numpy(), O.dequantize(oq, os_, ob, 128, bits))
        assert (x - xh).abs().max().item() <= 127.0 / (1 << bits)


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_quantize_mlx_edge_groups_bitexact(bits):
    """MLX's affine quantiser on the GPU: groups that are all zero, constant,
    one-signed, spanning zero or with |min| == |max|, in bf16 and f32, equal
    the oracle byte for byte; the scale's sign follows the larger-magnitude
    end and the bias is that end (or 0)."""
    from mlxr_moe import ops

    w = O.bf16_to_f32(O.normal_bf16(0, 170 + bits, (32, 256), 0.02)).copy()
    w[0, :64] = 0.0
    w[1, :64] = 0.03125
    w[2, :64] = -np.abs(w[2, :64])
    w[3, :64] = np.abs(w[3, :64])
    w[4, :64] = np.linspace(-0.5, 0.5, 64)
    w[5, :64] = np.linspace(-1.0, 0.875, 64)
    w[5, 1] = 0.0
    wb = O.f32_to_bf16(w.astype(np.float32))
    for host in (wb, O.bf16_to_f32(wb).astype(np.float32)):
        dev = np_bf16_to_torch(host) if host.dtype == np.uint16 else torch.from_numpy(host).cuda()
        wq, s, b = ops.quantize(dev, 64, bits)
        oq, os_, ob = O.quantize(host, 64, bits)
        np.testing.assert_array_equal(u32(wq), oq)
        if host.dtype == np.uint16:
            np.testing.assert_array_equal(bf16_np(s), os_)
            np.testing.assert_array_equal(bf16_np(b), ob)
            sf, bf = to_f32(os_), to_f32(ob)
        else:
            np.testing.assert_array_equal(s.cpu().numpy(), os_)
            np.testing.assert_array_equal(b.cpu().numpy(), ob)
            sf, bf = os_, ob
        g = O.bf16_to_f32(wb).reshape(32, 4, 64)
        mn, mx = g.min(-1), g.max(-1)
        assert ((sf < 0) == (np.abs(mx) >= np.abs(mn))).all()
        edge = np.where(np.abs(mn) > np.abs(mx), mn, mx)
        assert ((bf == edge) | (bf == 0)).all()


def test_dequantize_bf16_out_bitexact():
    from mlxr_moe import ops

    w = ops.synth_normal_bf16(0, 50, (64, 512), 0.02)
    wq, s, b = ops.quantize(w, 64, 4)
    d = ops.dequantize(wq, s, b, 64, 4)
    want = O.dequantize(u32(wq), bf16_np(s), bf16_np(b), 64, 4, out_dtype=np.uint16)
    np.testing.assert_array_equal(bf16_np(d), want)


def test_quantized_matmul_reference_relation():
    """quantization.rs:318-341: qmm == x @ dequant(w) within 1e-3 (transpose=false)."""
    from mlxr_moe import ops

    m, n, k = 32, 128, 128
    x = (ops.synth_normal_bf16(0, 60, (m, k), 1.0).float() / np.sqrt(k)).contiguous()
    w = (ops.synth_normal_bf16(0, 61, (k, n), 1.0).float() / np.sqrt(k)).contiguous()
    wq, s, b = ops.quantize(w, 64, 4)
    wh = ops.dequantize(wq, s, b, 64, 4)
    y = ops.quantized_matmul(x, wq, s, b, False, 64, 4)
    assert (y - x @ wh).abs().max().item() < 1e-3
    yo = O.quantized_matmul(x.cpu().numpy(), u32(wq), s.cpu().numpy(), b.cpu().numpy(), False, 64, 4)
    assert np.abs(y.cpu().numpy() - yo).max() < 1e-3
    # transpose=true (QuantizedLinear::forward) on bf16
    xb = ops.synth_normal_bf16(0, 62, (5, 256), 1.0)
    wt = ops.synth_normal_bf16(0, 63, (384, 256), 0.02)
    tq, ts, tb = ops.quantize(wt, 64, 8)
    yt = ops.quantized_matmul(xb, tq, ts, tb, True, 64, 8)
    yo = O.quantized_matmul(bf16_np(xb), u32(tq), bf16_np(ts), bf16_np(tb), True, 64, 8)
    assert np.abs(yt.float().cpu().numpy() - yo).max() < 1e-2


def test_gather_qmm_reference_cases():
    """quantization.rs:344-421: gather_qmm == gather_mm on dequantised weights (1e-4, f32)."""
    from mlxr_moe import ops

    m, n, k = 32, 64, 64
    w = ops.synth_normal_bf16(0, 70, (3, n, k), 1.0).float()
    wq, s, b = ops.quantize(w, 64, 4)
    w_hat = ops.dequantize(wq, s, b, 64, 4).transpose(-1, -2).contiguous()
    rhs = torch.tensor([2, 1], dtype=torch.int32, device="cuda")
    for xb, lhs in ((1, torch.tensor([0], dtype=torch.int32, device="cuda")),
                    (5, torch.tensor([0, 2], dtype=torch.int32, device="cuda"))):
        x = ops.synth_normal_bf16(0, 71 + xb, (xb, m, k), 1.0).float()
        c1 = ops.gather_mm(x, w_hat, lhs, rhs)
        c2 = ops.gather_qmm(x, wq, s, b, lhs, rhs, True, 64, 4)
        assert torch.allclose(c1, c2, rtol=1e-4, atol=1e-4)
        c3 = O.gather_qmm(x.cpu().numpy(), u32(wq), s.cpu().numpy(), b.cpu().numpy(),
                          lhs.expand(2).cpu().numpy(), rhs.cpu().numpy(), True, 64, 4)
        np.testing.assert_allclose(c2.cpu().numpy(), c3, rtol=1e-4, atol=1e-4)


def test_gather_qmm_moe_shape_and_sorted_flag():
    """The switch-layer call shape: x [T,1,1,D], rhs [T,K] -> [T,K,1,N] (switch.rs:148-167)."""
    from mlxr_moe import ops

    T, K, E, D, N = 24, 4, 8, 512, 256
    x = ops.synth_normal_bf16(0, 80, (T, 1, 1, D), 1.0)
    w = ops.synth_normal_bf16(0, 81, (E, N, D), 0.02)
    wq, s, b = ops.quantize(w, 64, 4)
    idx = (torch.arange(T * K, device="cuda", dtype=torch.int32) * 7 % E).reshape(T, K)
    y = ops.gather_qmm(x, wq, s, b, None, idx, True, 64, 4)
    assert tuple(y.shape) == (T, K, 1, N)
    yo = O.gather_qmm(bf16_np(x).reshape(T, 1, D), u32(wq), bf16_np(s), bf16_np(b),
                      np.repeat(np.arange(T), K).astype(np.int32), idx.reshape(-1).cpu().numpy(), True, 64, 4)
    np.testing.assert_allclose(y.float().reshape(T * K, N).cpu().numpy(), yo.reshape(T * K, N), atol=2e-2, rtol=1e-2)
    ys = ops.gather_qmm(x, wq, s, b, None, idx, True, 64, 4, sorted_indices=True)
    assert torch.equal(y, ys)


def test_gather_mm_reference_cases():
    from mlxr_moe import ops

    a = ops.synth_normal_bf16(0, 90, (1, 32, 32), 1.0).float()
    b = ops.synth_normal_bf16(0, 91, (3, 32, 32), 1.0).float()
    rhs = torch.tensor([2, 1], dtype=torch.int32, device="cuda")
    out = ops.gather_mm(a, b, torch.tensor([0], dtype=torch.int32, device="cuda"), rhs)
    ref = torch.stack([a[0] @ b[2], a[0] @ b[1]])
    assert torch.allclose(out, ref, rtol=1e-5, atol=1e-5)
    out = ops.gather_mm(a, b, None, rhs)
    assert torch.allclose(out, ref, rtol=1e-5, atol=1e-5)
    a100 = ops.synth_normal_bf16(0, 92, (100, 1, 100), 1.0).float()
    b8 = ops.synth_normal_bf16(0, 93, (8, 100, 100), 1.0).float()
    r = torch.sort(torch.arange(100, device="cuda", dtype=torch.int32) * 13 % 8).values.to(torch.int32)
    out = ops.gather_mm(a100, b8, None, r, sorted_indices=True)
    ref = torch.stack([a100[i] @ b8[r[i]] for i in range(100)])
    assert torch.allclose(out, ref, rtol=1e-4, atol=1e-4)


def test_out_of_range_index_reports_status():
    from mlxr_moe import MlxrError, _lib, ops

    ops.op_status()  # clear
    x = ops.synth_normal_bf16(0, 95, (1, 4, 64), 1.0)
    w = ops.synth_normal_bf16(0, 96, (3, 64, 64), 0.02)
    wq, s, b = ops.quantize(w, 64, 4)
    bad = torch.tensor([5], dtype=torch.int32, device="cuda")
    ops.gather_qmm(x, wq, s, b, None, bad, True, 64, 4)
    with pytest.raises(MlxrError) as ei:
        ops.op_status()
    assert ei.value.status == _lib.ERR_DEVICE_INDEX
    ops.op_status()  # cleared by the read


def _ws_bytes(ops, x_batch, M, K, w_batch, N, P, bits):
    import ctypes as C

    from mlxr_moe import _lib

    n = C.c_size_t(0)
    _lib.call("mlxr_cu_gather_qmm_workspace_size", 0, x_batch, M, K, w_batch, N, P, 1, 64, bits, C.byref(n))
    return n.value


@pytest.mark.parametrize("bits", [4, 8])
def test_gather_qmm_tensor_core_path_vs_oracle(bits):
    """The tensor-core gather_qmm (counting sort by rhs, gather of x[lhs], the
    grouped tcgen05 GEMM, write-back in index order) on unsorted rhs with lhs
    indices and M > 1 rows per index, against the oracle (fp32 accumulation;
    bf16 output and bf16-dequantised weights: |err| < 2e-2 + 1e-2 |ref|) and
    against the general CUDA-core kernel."""
    from mlxr_moe import ops

    xb, M, K, E, N, P = 6, 3, 512, 12, 384, 40
    assert _ws_bytes(ops, xb, M, K, E, N, P, bits) > 0
    x = ops.synth_normal_bf16(0, 100 + bits, (xb, M, K), 1.0)
    w = ops.synth_normal_bf16(0, 110 + bits, (E, N, K), 0.05)
    wq, s, b = ops.quantize(w, 64, bits)
    g = torch.Generator().manual_seed(bits)
    lhs = torch.randint(0, xb, (P,), generator=g, dtype=torch.int32).cuda()
    rhs = torch.randint(0, E, (P,), generator=g, dtype=torch.int32).cuda()
    y = ops.gather_qmm(x, wq, s, b, lhs, rhs, True, 64, bits)
    assert tuple(y.shape) == (P, M, N)
    yo = O.gather_qmm(bf16_np(x), u32(wq), bf16_np(s), bf16_np(b), lhs.cpu().numpy(), rhs.cpu().numpy(), True, 64,
                      bits)
    np.testing.assert_allclose(y.float().cpu().numpy(), yo, atol=2e-2, rtol=1e-2)
    yg = ops.gather_qmm_general(x, wq, s, b, lhs, rhs, True, 64, bits)
    np.testing.assert_allclose(y.float().cpu().numpy(), yg.float().cpu().numpy(), atol=2e-2, rtol=1e-2)
    ops.op_status()


def test_gather_qmm_tensor_core_path_moe_sized():
    """A switch-layer sized call (T=512 tokens, top-8 of 64 experts, D=1024,
    N=768) through the tensor-core path against the oracle."""
    from mlxr_moe import ops

    T, Kt, E, D, N = 512, 8, 64, 1024, 768
    x = ops.synth_normal_bf16(0, 120, (T, 1, 1, D), 1.0)
    w = ops.synth_normal_bf16(0, 121, (E, N, D), 0.03)
    wq, s, b = ops.quantize(w, 64, 4)
    g = torch.Generator().manual_seed(7)
    idx = torch.stack([torch.randperm(E, generator=g)[:Kt] for _ in range(T)]).to(torch.int32).cuda()
    y = ops.gather_qmm(x, wq, s, b, None, idx, True, 64, 4)
    assert tuple(y.shape) == (T, Kt, 1, N)
    yo = O.gather_qmm(bf16_np(x).reshape(T, 1, D), u32(wq), bf16_np(s), bf16_np(b),
                      np.repeat(np.arange(T), Kt).astype(np.int32), idx.reshape(-1).cpu().numpy(), True, 64, 4)
    np.testing.assert_allclose(y.float().reshape(T * Kt, N).cpu().numpy(), yo.reshape(T * Kt, N), atol=2e-2,
                               rtol=1e-2)
    ops.op_status()


@pytest.mark.parametrize("bits", [4, 8])
def test_quantized_matmul_tensor_core_path(bits):
    """QuantizedLinear::forward shape (transpose, bf16) on the tensor-core
    path: M = 300 rows (two partial 128-row tiles) against the oracle."""
    from mlxr_moe import ops

    M, K, N = 300, 768, 512
    assert _ws_bytes(ops, 1, M, K, 1, N, 1, bits) > 0
    x = ops.synth_normal_bf16(0, 130 + bits, (M, K), 1.0)
    w = ops.synth_normal_bf16(0, 140 + bits, (N, K), 0.04)
    wq, s, b = ops.quantize(w, 64, bits)
    y = ops.quantized_matmul(x, wq, s, b, True, 64, bits)
    yo = O.quantized_matmul(bf16_np(x), u32(wq), bf16_np(s), bf16_np(b), True, 64, bits)
    np.testing.assert_allclose(y.float().cpu().numpy(), yo, atol=2e-2, rtol=1e-2)
    ops.op_status()


def test_gather_qmm_tensor_core_path_bad_index_status():
    """An out-of-range rhs index on the tensor-core path: the row is skipped
    and the op status word reports it."""
    from mlxr_moe import MlxrError, _lib, ops

    ops.op_status()
    x = ops.synth_normal_bf16(0, 150, (4, 1, 256), 1.0)
    w = ops.synth_normal_bf16(0, 151, (3, 128, 256), 0.02)
    wq, s, b = ops.quantize(w, 64, 4)
    assert _ws_bytes(ops, 4, 1, 256, 3, 128, 4, 4) > 0
    bad = torch.tensor([0, 7, 1, 2], dtype=torch.int32, device="cuda")
    ops.gather_qmm(x, wq, s, b, None, bad, True, 64, 4)
    with pytest.raises(MlxrError) as ei:
        ops.op_status()
    assert ei.value.status == _lib.ERR_DEVICE_INDEX
    ops.op_status()
