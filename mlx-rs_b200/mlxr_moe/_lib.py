"""ctypes binding of libmlxr_moe.so (the C ABI declared in include/mlxr_moe.h).

The status/last-error contract mirrors the reference's Guarded::try_from_op
(crates/mlxr/src/utils/guard.rs:31-51): a non-zero status raises MlxrError
carrying the thread-local message (crates/mlxr/src/error.rs:229-290).

There is no fallback: if the shared library is missing or cannot be loaded,
importing this module raises.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(_HERE), "libmlxr_moe.so")

OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_UNSUPPORTED = 2
ERR_CUDA = 3
ERR_WORKSPACE = 4
ERR_TIMEOUT = 5
ERR_NCCL = 6
ERR_DEVICE_INDEX = 7

BFLOAT16, FLOAT16, FLOAT32 = 0, 1, 2

# Every entry point include/mlxr_moe.h declares.
EXPORTS = (
    "mlxr_cu_last_error",
    "mlxr_cu_clear_error",
    "mlxr_cu_abi_version",
    "mlxr_cu_quantize",
    "mlxr_cu_dequantize",
    "mlxr_cu_quantized_matmul",
    "mlxr_cu_gather_qmm",
    "mlxr_cu_gather_qmm_workspace_size",
    "mlxr_cu_gather_qmm_ws",
    "mlxr_cu_quantized_matmul_ws",
    "mlxr_cu_gather_mm",
    "mlxr_cu_moe_workspace_size",
    "mlxr_cu_moe_block_forward",
    "mlxr_cu_moe_block_forward_noalloc",
    "mlxr_cu_moe_status",
    "mlxr_cu_moe_set_stage_events",
    "mlxr_cu_op_status",
    "mlxr_cu_moe_router",
    "mlxr_cu_moe_permute",
    "mlxr_cu_moe_experts",
    "mlxr_cu_moe_combine",
    "mlxr_cu_synth_normal_bf16",
    "mlxr_cu_moe_ep_workspace_size",
    "mlxr_cu_moe_ep_dispatch",
    "mlxr_cu_moe_ep_experts",
    "mlxr_cu_moe_ep_combine",
    "mlxr_cu_ep_comm_create",
    "mlxr_cu_ep_comm_connect",
    "mlxr_cu_ep_comm_destroy",
    "mlxr_cu_moe_ep_p2p_workspace_size",
    "mlxr_cu_moe_ep_dispatch_p2p",
    "mlxr_cu_moe_ep_experts_p2p",
    "mlxr_cu_moe_ep_combine_p2p",
)


class MlxrError(RuntimeError):
    """A non-zero status from the C ABI, with the library's message."""

    def __init__(self, status: int, what: str):
        super().__init__(f"[status {status}] {what}")
        self.status = status
        self.what = what


P = C.c_void_p
I64 = C.c_int64
I32 = C.c_int


class QLinear(C.Structure):
    _fields_ = [("weight", P), ("scales", P), ("biases", P)]


class MoeConfig(C.Structure):
    _fields_ = [
        ("hidden_size", I32),
        ("num_experts", I32),
        ("num_experts_per_tok", I32),
        ("moe_intermediate_size", I32),
        ("shared_expert_intermediate_size", I32),
        ("group_size", I32),
        ("bits", I32),
        ("shared_bits", I32),
        ("norm_topk_prob", I32),
        ("shared_gate_bits", I32),
        ("model_kind", I32),
        ("rms_norm_eps", C.c_float),
    ]


class MoeWeights(C.Structure):
    _fields_ = [
        ("router_weight", P),
        ("router_bias", P),
        ("switch_gate", QLinear),
        ("switch_up", QLinear),
        ("switch_down", QLinear),
        ("shared_gate", QLinear),
        ("shared_up", QLinear),
        ("shared_down", QLinear),
        ("shared_expert_gate", QLinear),
        ("switch_gate_up", QLinear),
        ("router_norm", P),
        ("expert_scale", P),
        ("experts_norm", P),
    ]


class MoeRouting(C.Structure):
    _fields_ = [
        ("indices", P),
        ("weights", P),
        ("counts", P),
        ("offsets", P),
        ("sorted_rows", P),
        ("inverse", P),
    ]


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python mlx-rs_b200/build.py` "
            "(there is no CPU fallback for this library)"
        )
    lib = C.CDLL(LIB_PATH)
    for name in EXPORTS:
        getattr(lib, name)  # raises AttributeError if a symbol is missing
    lib.mlxr_cu_last_error.restype = C.c_char_p
    lib.mlxr_cu_last_error.argtypes = []
    lib.mlxr_cu_clear_error.restype = None
    lib.mlxr_cu_abi_version.restype = I32
    lib.mlxr_cu_quantize.argtypes = [P, I32, I64, I64, I32, I32, C.c_char_p, P, P, P, P]
    lib.mlxr_cu_dequantize.argtypes = [P, P, P, I32, I64, I64, I32, I32, C.c_char_p, P, I32, P]
    lib.mlxr_cu_quantized_matmul.argtypes = [P, I32, I64, I64, P, P, P, I64, I32, I32, I32, C.c_char_p, P, P]
    lib.mlxr_cu_gather_qmm.argtypes = [P, I32, I64, I64, I64, P, P, P, I64, I64, P, P, I64, I32, I32, I32,
                                       C.c_char_p, I32, P, P]
    lib.mlxr_cu_gather_qmm_workspace_size.argtypes = [I32, I64, I64, I64, I64, I64, I64, I32, I32, I32,
                                                      C.POINTER(C.c_size_t)]
    lib.mlxr_cu_gather_qmm_ws.argtypes = [P, I32, I64, I64, I64, P, P, P, I64, I64, P, P, I64, I32, I32, I32,
                                          C.c_char_p, I32, P, P, C.c_size_t, P]
    lib.mlxr_cu_quantized_matmul_ws.argtypes = [P, I32, I64, I64, P, P, P, I64, I32, I32, I32, C.c_char_p, P, P,
                                                C.c_size_t, P]
    lib.mlxr_cu_gather_mm.argtypes = [P, P, I32, I64, I64, I64, I64, I64, P, P, I64, I32, P, P]
    lib.mlxr_cu_moe_workspace_size.argtypes = [C.POINTER(MoeConfig), I64, C.POINTER(C.c_size_t)]
    lib.mlxr_cu_moe_block_forward.argtypes = [C.POINTER(MoeConfig), C.POINTER(MoeWeights), P, I64, P,
                                              C.POINTER(MoeRouting), P, C.c_size_t, P]
    lib.mlxr_cu_moe_block_forward_noalloc.argtypes = [C.POINTER(MoeConfig), C.POINTER(MoeWeights), P, I64, P,
                                                      C.POINTER(MoeRouting), P, P]
    lib.mlxr_cu_moe_status.argtypes = [P, P]
    lib.mlxr_cu_moe_set_stage_events.argtypes = [C.POINTER(C.c_void_p), I32]
    lib.mlxr_cu_op_status.argtypes = [P]
    lib.mlxr_cu_moe_router.argtypes = [C.POINTER(MoeConfig), C.POINTER(MoeWeights), P, I64, P, P, P, P, P,
                                       C.c_size_t, P]
    lib.mlxr_cu_moe_permute.argtypes = [C.POINTER(MoeConfig), P, I64, P, P, P, P, P, P, P, C.c_size_t, P]
    lib.mlxr_cu_moe_experts.argtypes = [C.POINTER(MoeConfig), C.POINTER(MoeWeights), P, I64, P, P, P, C.c_size_t, P]
    lib.mlxr_cu_moe_combine.argtypes = [C.POINTER(MoeConfig), C.POINTER(MoeWeights), P, I64, P, P, P, P, P,
                                        C.c_size_t, P]
    lib.mlxr_cu_synth_normal_bf16.argtypes = [C.c_uint64, C.c_uint64, I64, C.c_float, P, P]
    cfg_p, w_p = C.POINTER(MoeConfig), C.POINTER(MoeWeights)
    lib.mlxr_cu_moe_ep_workspace_size.argtypes = [cfg_p, I32, I64, I64, I64, C.POINTER(C.c_size_t)]
    lib.mlxr_cu_moe_ep_dispatch.argtypes = [cfg_p, w_p, I32, P, P, I64, P, P, P, P, P, P, C.c_size_t, P]
    lib.mlxr_cu_moe_ep_experts.argtypes = [cfg_p, w_p, I32, P, P, I64, I64, P, P, C.c_size_t, P]
    lib.mlxr_cu_moe_ep_combine.argtypes = [cfg_p, w_p, P, I64, P, I64, P, P, P, P, C.c_size_t, P]
    U32 = C.c_uint32
    lib.mlxr_cu_ep_comm_create.argtypes = [I32, I32, I64, I32, I32, C.POINTER(C.c_void_p), P]
    lib.mlxr_cu_ep_comm_connect.argtypes = [P, P]
    lib.mlxr_cu_ep_comm_destroy.argtypes = [P]
    lib.mlxr_cu_moe_ep_p2p_workspace_size.argtypes = [cfg_p, P, I64, I32, I64, C.POINTER(C.c_size_t)]
    lib.mlxr_cu_moe_ep_dispatch_p2p.argtypes = [cfg_p, w_p, P, P, P, I64, P, P, U32, P, C.c_size_t, P]
    lib.mlxr_cu_moe_ep_experts_p2p.argtypes = [cfg_p, w_p, I32, P, I64, U32, P, C.c_size_t, P]
    lib.mlxr_cu_moe_ep_combine_p2p.argtypes = [cfg_p, w_p, P, P, I64, P, P, P, U32, P, C.c_size_t, P]
    for name in EXPORTS:
        f = getattr(lib, name)
        if f.restype is C.c_int or name not in ("mlxr_cu_last_error", "mlxr_cu_clear_error"):
            if name not in ("mlxr_cu_last_error", "mlxr_cu_clear_error"):
                f.restype = I32
    return lib


LIB = _load()


def last_error() -> str | None:
    m = LIB.mlxr_cu_last_error()
    return None if m is None else m.decode("utf-8", "replace")


def check(status: int) -> None:
    """Guarded::try_from_op: 0 is success, otherwise raise with the message."""
    if status != OK:
        msg = last_error() or "operation failed but no error was set"
        LIB.mlxr_cu_clear_error()
        raise MlxrError(status, msg)


def call(name: str, *args) -> None:
    check(getattr(LIB, name)(*args))
