"""ctypes wrapper over the CPU oracle (``liboracle.so``).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py``, never by
the product package. Parity against the reference's own outputs is unpinned
(MLX, which holds the reference's arithmetic, is not buildable here); the
oracle restates the reference's dataflow and is pinned by the relations the
reference's own tests assert. Each function names the reference code it
restates.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

DT_BF16, DT_F16, DT_F32 = 0, 1, 2


def build(force: bool = False) -> str:
    """Compile liboracle.so with the committed Makefile (checker, not product)."""
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(
        os.path.join(_HERE, "moe_oracle.cpp")
    ):
        subprocess.run(["make", "-C", _HERE, "-s"], check=True)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = C.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


P = C.c_void_p
I64 = C.c_int64
I32 = C.c_int


class OrcQuant(C.Structure):
    _fields_ = [("w", P), ("s", P), ("b", P)]


class OrcMoeConfig(C.Structure):
    _fields_ = [
        ("hidden", I32),
        ("num_experts", I32),
        ("top_k", I32),
        ("moe_intermediate", I32),
        ("shared_intermediate", I32),
        ("group_size", I32),
        ("bits", I32),
        ("shared_bits", I32),
        ("renorm", I32),
        ("shared_gate_bits", I32),
    ]


class OrcMoeWeights(C.Structure):
    _fields_ = [
        ("router", P),
        ("router_bias", P),
        ("gate", OrcQuant),
        ("up", OrcQuant),
        ("down", OrcQuant),
        ("sh_gate", OrcQuant),
        ("sh_up", OrcQuant),
        ("sh_down", OrcQuant),
        ("sh_expert_gate", OrcQuant),
    ]


class OrcGemma4Config(C.Structure):
    _fields_ = [
        ("hidden", I32),
        ("num_experts", I32),
        ("top_k", I32),
        ("moe_intermediate", I32),
        ("group_size", I32),
        ("bits", I32),
        ("eps", C.c_float),
    ]


class OrcGemma4Weights(C.Structure):
    _fields_ = [
        ("router", P),
        ("router_norm", P),
        ("expert_scale", P),
        ("experts_norm", P),
        ("gate_up", OrcQuant),
        ("down", OrcQuant),
    ]


def _declare(L):
    L.orc_normal_bf16.argtypes = [C.c_uint64, C.c_uint64, I64, C.c_float, P]
    L.orc_normal_bf16.restype = None
    L.orc_f32_to_bf16.argtypes = [P, I64, P]
    L.orc_exp_route.argtypes = [P, I64, P]
    L.orc_dot_rn32.argtypes = [P, P, I64, I32, P]
    L.orc_quantize.argtypes = [P, I32, I64, I64, I32, I32, P, P, P]
    L.orc_dequantize.argtypes = [P, P, P, I32, I64, I64, I32, I32, P, I32]
    L.orc_gather_qmm.argtypes = [P, I32, I64, I64, I64, P, P, P, I32, I64, I64, P, P, I64, I32, I32, I32, P]
    L.orc_quantized_matmul.argtypes = [P, I32, I64, I64, P, P, P, I32, I64, I32, I32, I32, P]
    L.orc_gather_mm.argtypes = [P, I64, I64, I64, P, I64, I64, P, P, I64, P]
    L.orc_router.argtypes = [P, I64, I32, P, I32, P, I32, I32, P, P, P, P]
    L.orc_permute.argtypes = [P, I64, I32, I32, P, P, P, P]
    L.orc_moe_block.argtypes = [C.POINTER(OrcMoeConfig), C.POINTER(OrcMoeWeights), P, I64, I32, P, P, P]
    L.orc_gemma4_block.argtypes = [C.POINTER(OrcGemma4Config), C.POINTER(OrcGemma4Weights), P, I64, P, P, P]
    L.orc_set_threads.argtypes = [I32]
    L.orc_max_threads.restype = I32


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _dt(a: np.ndarray) -> int:
    if a.dtype == np.float32:
        return DT_F32
    if a.dtype == np.float16:
        return DT_F16
    if a.dtype == np.uint16:  # bf16 bit patterns
        return DT_BF16
    raise TypeError(f"unsupported dtype {a.dtype}")


# ------------------------------------------------------------- helpers ----
def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty(a.shape, np.uint16)
    lib().orc_f32_to_bf16(_p(a), a.size, _p(out))
    return out


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def max_threads() -> int:
    return int(lib().orc_max_threads())


def normal_bf16(seed: int, stream: int, shape, stddev: float) -> np.ndarray:
    n = int(np.prod(shape))
    out = np.empty(n, np.uint16)
    lib().orc_normal_bf16(seed, stream, n, stddev, _p(out))
    return out.reshape(shape)


def exp_route(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    lib().orc_exp_route(_p(x), x.size, _p(out))
    return out


def dot_rn32(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """Row-wise exact dot products of bf16 bit arrays [rows, D], each rounded
    once to fp32 (the router logit's sum)."""
    x = np.ascontiguousarray(x, np.uint16)
    w = np.ascontiguousarray(w, np.uint16)
    assert x.shape == w.shape and x.ndim == 2
    out = np.empty(x.shape[0], np.float32)
    lib().orc_dot_rn32(_p(x), _p(w), x.shape[0], x.shape[1], _p(out))
    return out


# ------------------------------------------------------- op family -------
def quantize(w: np.ndarray, group_size: int = 64, bits: int = 4):
    """quantization.rs:47 (mode affine): w [..., cols] -> (wq u32, scales, biases)."""
    w = np.ascontiguousarray(w)
    cols = w.shape[-1]
    rows = w.size // cols
    wq = np.empty(w.shape[:-1] + (cols * bits // 32,), np.uint32)
    s = np.empty(w.shape[:-1] + (cols // group_size,), w.dtype)
    b = np.empty_like(s)
    rc = lib().orc_quantize(_p(w), _dt(w), rows, cols, group_size, bits, _p(wq), _p(s), _p(b))
    if rc:
        raise ValueError(f"orc_quantize rc={rc}")
    return wq, s, b


def dequantize(wq, scales, biases, group_size: int = 64, bits: int = 4, out_dtype=np.float32):
    """quantization.rs:118: -> [..., cols] in out_dtype (np.uint16 = bf16)."""
    cols = wq.shape[-1] * 32 // bits
    rows = wq.size // wq.shape[-1]
    out = np.empty(wq.shape[:-1] + (cols,), out_dtype)
    rc = lib().orc_dequantize(
        _p(np.ascontiguousarray(wq)), _p(np.ascontiguousarray(scales)), _p(np.ascontiguousarray(biases)),
        _dt(scales), rows, cols, group_size, bits, _p(out), _dt(out),
    )
    if rc:
        raise ValueError(f"orc_dequantize rc={rc}")
    return out


def gather_qmm(x, wq, scales, biases, lhs=None, rhs=None, transpose=True, group_size=64, bits=4):
    """quantization.rs:171 with flattened indices: x [xb, M, K] -> [P, M, N] fp32."""
    x = np.ascontiguousarray(x)
    xb, M, K = x.shape
    wb = wq.shape[0]
    if transpose:
        N = wq.shape[1]
    else:
        N = wq.shape[2] * 32 // bits
    if lhs is None and rhs is None:
        Pn = max(xb, wb)
    else:
        Pn = len(lhs) if lhs is not None else len(rhs)
    lhs_a = None if lhs is None else np.ascontiguousarray(lhs, np.int32)
    rhs_a = None if rhs is None else np.ascontiguousarray(rhs, np.int32)
    out = np.empty((Pn, M, N), np.float32)
    rc = lib().orc_gather_qmm(
        _p(x), _dt(x), xb, M, K, _p(np.ascontiguousarray(wq)), _p(np.ascontiguousarray(scales)),
        _p(np.ascontiguousarray(biases)), _dt(scales), wb, N, _p(lhs_a), _p(rhs_a), Pn, int(transpose),
        group_size, bits, _p(out),
    )
    if rc:
        raise ValueError(f"orc_gather_qmm rc={rc}")
    return out


def quantized_matmul(x, wq, scales, biases, transpose=True, group_size=64, bits=4):
    """quantization.rs:81: x [M, K] -> [M, N] fp32."""
    x = np.ascontiguousarray(x)
    M, K = x.shape
    N = wq.shape[0] if transpose else wq.shape[1] * 32 // bits
    out = np.empty((M, N), np.float32)
    rc = lib().orc_quantized_matmul(
        _p(x), _dt(x), M, K, _p(np.ascontiguousarray(wq)), _p(np.ascontiguousarray(scales)),
        _p(np.ascontiguousarray(biases)), _dt(scales), N, int(transpose), group_size, bits, _p(out),
    )
    if rc:
        raise ValueError(f"orc_quantized_matmul rc={rc}")
    return out


def gather_mm(a, b, lhs=None, rhs=None):
    """arithmetic.rs:1577: a [ab, M, K] f32, b [bb, K, N] f32 -> [P, M, N]."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    ab, M, K = a.shape
    bb, _, N = b.shape
    Pn = len(lhs) if lhs is not None else (len(rhs) if rhs is not None else max(ab, bb))
    lhs_a = None if lhs is None else np.ascontiguousarray(lhs, np.int32)
    rhs_a = None if rhs is None else np.ascontiguousarray(rhs, np.int32)
    out = np.empty((Pn, M, N), np.float32)
    rc = lib().orc_gather_mm(_p(a), ab, M, K, _p(b), bb, N, _p(lhs_a), _p(rhs_a), Pn, _p(out))
    if rc:
        raise ValueError(f"orc_gather_mm rc={rc}")
    return out


# ------------------------------------------------------------ routing ----
def router(x, wg, top_k, bias=None, renorm=True, want_logits=False):
    """moe.rs:123-138 under the routing contract. x [T, D] bf16, wg [E, D] bf16."""
    x = np.ascontiguousarray(x, np.uint16)
    wg = np.ascontiguousarray(wg, np.uint16)
    T, D = x.shape
    E = wg.shape[0]
    idx = np.empty((T, top_k), np.int32)
    w = np.empty((T, top_k), np.uint16)
    lg = np.empty((T, E), np.uint16) if want_logits else None
    pr = np.empty((T, E), np.uint16) if want_logits else None
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    rc = lib().orc_router(_p(x), T, D, _p(wg), E, _p(b), top_k, int(renorm), _p(idx), _p(w), _p(lg), _p(pr))
    if rc:
        raise ValueError(f"orc_router rc={rc}")
    if want_logits:
        return idx, w, lg, pr
    return idx, w


def permute(idx, num_experts):
    """switch.rs:499-517 stable sort by expert: (counts, offsets, sorted_flat, inv)."""
    idx = np.ascontiguousarray(idx, np.int32)
    T, K = idx.shape
    counts = np.empty(num_experts, np.int32)
    offsets = np.empty(num_experts + 1, np.int32)
    sorted_flat = np.empty(T * K, np.int32)
    inv = np.empty(T * K, np.int32)
    rc = lib().orc_permute(_p(idx), T, K, num_experts, _p(counts), _p(offsets), _p(sorted_flat), _p(inv))
    if rc:
        raise ValueError(f"orc_permute rc={rc}")
    return counts, offsets, sorted_flat, inv


# -------------------------------------------------------------- block ----
def _q(t):
    if t is None:
        return OrcQuant(None, None, None)
    w, s, b = t
    return OrcQuant(_p(w), _p(s), _p(b))


def moe_block(cfg: dict, weights: dict, x: np.ndarray, mode: str = "fused"):
    """moe.rs:116-146. mode "staged" (MLX op-by-op bf16) or "fused" (kernel contract).

    weights: router [E,D] u16, router_bias [E] f32|None, gate/up/down/(sh_gate,
    sh_up, sh_down, sh_expert_gate) as (wq, scales, biases) triples.
    Returns (out [T,D] u16 bf16, idx [T,K] i32, w [T,K] u16 bf16).
    """
    x = np.ascontiguousarray(x, np.uint16)
    T = x.shape[0]
    c = OrcMoeConfig(
        cfg["hidden"], cfg["num_experts"], cfg["top_k"], cfg["moe_intermediate"], cfg.get("shared_intermediate", 0),
        cfg.get("group_size", 64), cfg.get("bits", 4), cfg.get("shared_bits", cfg.get("bits", 4)),
        int(cfg.get("renorm", True)), int(cfg.get("shared_gate_bits", 0) or 0),
    )
    keep = []

    def cont(a):
        if a is None:
            return None
        a = np.ascontiguousarray(a)
        keep.append(a)
        return a

    def trip(name):
        t = weights.get(name)
        if t is None:
            return None
        return tuple(cont(v) for v in t)

    w = OrcMoeWeights(
        _p(cont(weights["router"])), _p(cont(weights.get("router_bias"))), _q(trip("gate")), _q(trip("up")),
        _q(trip("down")), _q(trip("sh_gate")), _q(trip("sh_up")), _q(trip("sh_down")), _q(trip("sh_expert_gate")),
    )
    out = np.empty_like(x)
    idx = np.empty((T, c.top_k), np.int32)
    wk = np.empty((T, c.top_k), np.uint16)
    rc = lib().orc_moe_block(C.byref(c), C.byref(w), _p(x), T, 1 if mode == "fused" else 0, _p(out), _p(idx), _p(wk))
    if rc:
        raise ValueError(f"orc_moe_block rc={rc}")
    return out, idx, wk


def gemma4_block(cfg: dict, weights: dict, x: np.ndarray, routing_only: bool = False):
    """Gemma 4 MoE branch (gemma4/text/text.rs:622-664 router, text.rs:901-916
    experts on pre_feedforward_layernorm_2(h); nn/switch.rs:242-345 packed
    gate_up_proj with GeGLU) in the kernels' fused-fp32 contract.

    cfg: hidden, num_experts, top_k, moe_intermediate, group_size, bits, eps.
    weights: router [E,D] u16, router_norm [D] u16 (Router.scale *
    hidden^-0.5), expert_scale [E] u16, experts_norm [D] u16, gate_up
    [E,2I,..] and down [E,D,..] as (wq, scales, biases) triples.
    Returns (out [T,D] u16 or None, idx [T,K] i32, w [T,K] u16).
    """
    x = np.ascontiguousarray(x, np.uint16)
    T = x.shape[0]
    c = OrcGemma4Config(cfg["hidden"], cfg["num_experts"], cfg["top_k"], cfg["moe_intermediate"],
                        cfg.get("group_size", 64), cfg.get("bits", 4), float(cfg.get("eps", 1e-6)))
    keep = []

    def cont(a):
        a = np.ascontiguousarray(a)
        keep.append(a)
        return a

    def trip(name):
        return tuple(cont(v) for v in weights[name])

    w = OrcGemma4Weights(_p(cont(weights["router"])), _p(cont(weights["router_norm"])),
                         _p(cont(weights["expert_scale"])), _p(cont(weights["experts_norm"])),
                         _q(None if routing_only else trip("gate_up")), _q(None if routing_only else trip("down")))
    out = None if routing_only else np.empty_like(x)
    idx = np.empty((T, c.top_k), np.int32)
    wk = np.empty((T, c.top_k), np.uint16)
    rc = lib().orc_gemma4_block(C.byref(c), C.byref(w), _p(x), T, _p(out) if out is not None else None, _p(idx), _p(wk))
    if rc:
        raise ValueError(f"orc_gemma4_block rc={rc}")
    return out, idx, wk
