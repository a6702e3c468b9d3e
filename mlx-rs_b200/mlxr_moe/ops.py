"""The quantised op family with the reference's Python-visible semantics.

Mirrors crates/mlxr/src/ops/quantization.rs (quantize l.47, quantized_matmul
l.81, dequantize l.118, gather_qmm l.171) and gather_mm
(crates/mlxr/src/ops/arithmetic.rs:1577): the same argument names, defaults
(group_size 64, bits 4, mode "affine"; quantized_matmul transpose=False,
gather_qmm transpose=True, sorted_indices=False) and index broadcasting
(absent lhs/rhs indices are the arange over the operand's batch, then both
are broadcast together). Tensors are torch CUDA tensors; every call runs the
CUDA library through its C ABI on the current stream.
"""
from __future__ import annotations

import ctypes as C
import math

import torch

from . import _lib

DEFAULT_GROUP_SIZE = 64
DEFAULT_BITS = 4

_DT = {torch.bfloat16: _lib.BFLOAT16, torch.float16: _lib.FLOAT16, torch.float32: _lib.FLOAT32}


def _dt(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise _lib.MlxrError(_lib.ERR_INVALID_ARGUMENT, f"unsupported dtype {t.dtype}") from None


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise _lib.MlxrError(_lib.ERR_INVALID_ARGUMENT, "tensors must live on a CUDA device")


def _ptr(t):
    return None if t is None else t.data_ptr()


def _mode(mode):
    return None if mode is None else mode.encode()


def quantize(w: torch.Tensor, group_size: int | None = None, bits: int | None = None, mode: str = "affine"):
    """(packed uint32 [..., cols*bits/32], scales [..., cols/gs], biases)."""
    gs = group_size or DEFAULT_GROUP_SIZE
    b = bits or DEFAULT_BITS
    _cuda(w)
    if w.ndim < 2:
        raise _lib.MlxrError(_lib.ERR_INVALID_ARGUMENT, "quantize needs at least 2 dimensions")
    w = w.contiguous()
    cols = w.shape[-1]
    rows = w.numel() // cols
    if (cols * b) % 32:
        raise _lib.MlxrError(_lib.ERR_INVALID_ARGUMENT, f"cols={cols} does not pack into uint32 at bits={b}")
    wq = torch.empty(w.shape[:-1] + (cols * b // 32,), dtype=torch.int32, device=w.device)
    s = torch.empty(w.shape[:-1] + (max(cols // gs, 1),), dtype=w.dtype, device=w.device)
    bi = torch.empty_like(s)
    _lib.call("mlxr_cu_quantize", _ptr(w), _dt(w), rows, cols, gs, b, _mode(mode), _ptr(wq), _ptr(s), _ptr(bi),
              _stream(w))
    return wq, s, bi


def dequantize(w, scales, biases=None, group_size: int | None = None, bits: int | None = None,
               mode: str = "affine", dtype: torch.dtype | None = None):
    gs = group_size or DEFAULT_GROUP_SIZE
    b = bits or DEFAULT_BITS
    _cuda(w, scales, biases)
    cols = w.shape[-1] * 32 // b
    rows = w.numel() // w.shape[-1]
    out = torch.empty(w.shape[:-1] + (cols,), dtype=dtype or scales.dtype, device=w.device)
    _lib.call("mlxr_cu_dequantize", _ptr(w.contiguous()), _ptr(scales.contiguous()),
              _ptr(None if biases is None else biases.contiguous()), _dt(scales), rows, cols, gs, b, _mode(mode),
              _ptr(out), _dt(out), _stream(w))
    return out


def quantized_matmul(x, w, scales, biases=None, transpose: bool = False, group_size: int | None = None,
                     bits: int | None = None, mode: str = "affine"):
    """x [..., K] @ dequant(w)^T (transpose) or @ dequant(w); out dtype = x dtype."""
    gs = group_size or DEFAULT_GROUP_SIZE
    b = bits or DEFAULT_BITS
    _cuda(x, w, scales, biases)
    x = x.contiguous()
    K = x.shape[-1]
    M = x.numel() // K
    N = w.shape[0] if transpose else w.shape[1] * 32 // b
    out = torch.empty(x.shape[:-1] + (N,), dtype=x.dtype, device=x.device)
    ws = _workspace(x, 1, M, K, 1, N, 1, transpose, gs, b)
    _lib.call("mlxr_cu_quantized_matmul_ws", _ptr(x), _dt(x), M, K, _ptr(w.contiguous()), _ptr(scales.contiguous()),
              _ptr(None if biases is None else biases.contiguous()), N, int(transpose), gs, b, _mode(mode),
              _ptr(out), _ptr(ws), 0 if ws is None else ws.numel(), _stream(x))
    return out


def _workspace(x, x_batch, M, K, w_batch, N, num_indices, transpose, gs, b):
    """Device workspace of the tensor-core gather_qmm path (None when the
    shape takes the general kernel)."""
    n = C.c_size_t(0)
    _lib.call("mlxr_cu_gather_qmm_workspace_size", _dt(x), x_batch, M, K, w_batch, N, num_indices, int(transpose),
              gs, b, C.byref(n))
    if n.value == 0:
        return None
    return torch.empty(int(n.value), dtype=torch.uint8, device=x.device)


def _broadcast_indices(lhs, rhs, bx, bw, device):
    nx = math.prod(bx) if bx else 1
    nw = math.prod(bw) if bw else 1
    if lhs is None:
        lhs = torch.arange(nx, device=device, dtype=torch.int32).reshape(bx if bx else ())
    if rhs is None:
        rhs = torch.arange(nw, device=device, dtype=torch.int32).reshape(bw if bw else ())
    shape = torch.broadcast_shapes(lhs.shape, rhs.shape)
    lf = lhs.to(torch.int32).expand(shape).reshape(-1).contiguous()
    rf = rhs.to(torch.int32).expand(shape).reshape(-1).contiguous()
    return lf, rf, tuple(shape), nx, nw


def gather_qmm(x, w, scales, biases=None, lhs_indices=None, rhs_indices=None, transpose: bool = True,
               group_size: int | None = None, bits: int | None = None, sorted_indices: bool = False,
               mode: str = "affine"):
    """out[idx] = x[lhs[idx]] @ dequant(w[rhs[idx]])^T; shape broadcast(lhs, rhs) + [M, N]."""
    gs = group_size or DEFAULT_GROUP_SIZE
    b = bits or DEFAULT_BITS
    _cuda(x, w, scales, biases, lhs_indices, rhs_indices)
    x = x.contiguous()
    M, K = x.shape[-2], x.shape[-1]
    N = w.shape[-2] if transpose else w.shape[-1] * 32 // b
    lf, rf, shape, nx, nw = _broadcast_indices(lhs_indices, rhs_indices, x.shape[:-2], w.shape[:-2], x.device)
    out = torch.empty(shape + (M, N), dtype=x.dtype, device=x.device)
    ws = _workspace(x, nx, M, K, nw, N, lf.numel(), transpose, gs, b)
    _lib.call("mlxr_cu_gather_qmm_ws", _ptr(x), _dt(x), nx, M, K, _ptr(w.contiguous()), _ptr(scales.contiguous()),
              _ptr(None if biases is None else biases.contiguous()), nw, N, _ptr(lf), _ptr(rf), lf.numel(),
              int(transpose), gs, b, _mode(mode), int(sorted_indices), _ptr(out), _ptr(ws),
              0 if ws is None else ws.numel(), _stream(x))
    return out


def gather_qmm_general(x, w, scales, biases=None, lhs_indices=None, rhs_indices=None, transpose: bool = True,
                       group_size: int | None = None, bits: int | None = None, sorted_indices: bool = False,
                       mode: str = "affine"):
    """gather_qmm through the general CUDA-core kernel for every shape
    (mlxr_cu_gather_qmm, no workspace); the reference point of the tensor-core
    path's tests."""
    gs = group_size or DEFAULT_GROUP_SIZE
    b = bits or DEFAULT_BITS
    _cuda(x, w, scales, biases, lhs_indices, rhs_indices)
    x = x.contiguous()
    M, K = x.shape[-2], x.shape[-1]
    N = w.shape[-2] if transpose else w.shape[-1] * 32 // b
    lf, rf, shape, nx, nw = _broadcast_indices(lhs_indices, rhs_indices, x.shape[:-2], w.shape[:-2], x.device)
    out = torch.empty(shape + (M, N), dtype=x.dtype, device=x.device)
    _lib.call("mlxr_cu_gather_qmm", _ptr(x), _dt(x), nx, M, K, _ptr(w.contiguous()), _ptr(scales.contiguous()),
              _ptr(None if biases is None else biases.contiguous()), nw, N, _ptr(lf), _ptr(rf), lf.numel(),
              int(transpose), gs, b, _mode(mode), int(sorted_indices), _ptr(out), _stream(x))
    return out


def gather_mm(a, b, lhs_indices=None, rhs_indices=None, sorted_indices: bool = False):
    """out[idx] = a[lhs[idx]] @ b[rhs[idx]]; shape broadcast(lhs, rhs) + [M, N]."""
    _cuda(a, b, lhs_indices, rhs_indices)
    if a.dtype != b.dtype:
        raise _lib.MlxrError(_lib.ERR_INVALID_ARGUMENT, "gather_mm operands must share a dtype")
    a = a.contiguous()
    b = b.contiguous()
    M, K = a.shape[-2], a.shape[-1]
    N = b.shape[-1]
    lf, rf, shape, na, nb = _broadcast_indices(lhs_indices, rhs_indices, a.shape[:-2], b.shape[:-2], a.device)
    out = torch.empty(shape + (M, N), dtype=a.dtype, device=a.device)
    _lib.call("mlxr_cu_gather_mm", _ptr(a), _ptr(b), _dt(a), na, M, K, nb, N, _ptr(lf), _ptr(rf), lf.numel(),
              int(sorted_indices), _ptr(out), _stream(a))
    return out


def op_status(device=None) -> None:
    """Raise if an op-family kernel saw an index outside its batch since the last check."""
    st = torch.cuda.current_stream(device).cuda_stream
    _lib.call("mlxr_cu_op_status", st)


def synth_normal_bf16(seed: int, stream_id: int, shape, stddev: float, device="cuda") -> torch.Tensor:
    """Seeded N(0, stddev^2) bf16 tensor (Philox4x32-10 + Box-Muller)."""
    out = torch.empty(shape, dtype=torch.bfloat16, device=device)
    _lib.call("mlxr_cu_synth_normal_bf16", seed, stream_id, out.numel(), float(stddev), _ptr(out), _stream(out))
    return out
