"""B200 (sm_100a) MoE block and quantised op family for mlxr, over a C ABI.

Importing this package loads libmlxr_moe.so; it raises if the library is
missing (there is no CPU fallback).
"""
from . import _lib, checkpoint, ops, synth
from ._lib import MlxrError
from .checkpoint import load_gemma4_moe_branch, load_qwen35_moe_block
from .moe import (Gemma4MoeBranch, MoeConfig, PackedSwitchFfn, QuantizedLinear, QuantizedSwitchLinear,
                  Qwen35MoeBlock, Routing, SplitSwitchFfn, SwigluMlp)
from .ops import dequantize, gather_mm, gather_qmm, quantize, quantized_matmul

__all__ = [
    "Gemma4MoeBranch", "MlxrError", "MoeConfig", "PackedSwitchFfn", "QuantizedLinear", "QuantizedSwitchLinear", "Qwen35MoeBlock", "Routing",
    "SplitSwitchFfn", "SwigluMlp", "dequantize", "gather_mm", "gather_qmm", "quantize", "quantized_matmul",
    "ops", "synth", "_lib", "checkpoint", "load_qwen35_moe_block", "load_gemma4_moe_branch",
]
