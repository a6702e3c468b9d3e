"""CPU tests of the C-ABI boundary: the library loads, exports every entry
point include/mlxr_moe.h declares, and reports argument errors through the
status + thread-local message contract without touching a GPU."""
import ctypes as C
import os
import re
import subprocess

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "mlxr_moe.h")
LIB = os.path.join(ROOT, "mlx-rs_b200", "libmlxr_moe.so")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^MLXR_CU_API\s+[\w\s\*]+?\b(mlxr_cu_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    for s in ("mlxr_cu_gather_qmm", "mlxr_cu_quantized_matmul", "mlxr_cu_quantize", "mlxr_cu_dequantize",
              "mlxr_cu_moe_block_forward", "mlxr_cu_moe_workspace_size", "mlxr_cu_last_error"):
        assert s in syms


def test_library_exports_every_declared_symbol():
    assert os.path.exists(LIB), "build the library first (python mlx-rs_b200/build.py)"
    out = subprocess.run(["nm", "-D", "--defined-only", LIB], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (mlxr_cu_\w+)", out))
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, f"declared but not exported: {missing}"
    from mlxr_moe import _lib

    assert set(_lib.EXPORTS) == set(declared_symbols())


def test_abi_version_and_clean_error_state():
    from mlxr_moe import _lib

    assert _lib.LIB.mlxr_cu_abi_version() == 2
    _lib.LIB.mlxr_cu_clear_error()
    assert _lib.last_error() is None


def test_error_contract_workspace_size():
    """Invalid configs fail with status + message (Guarded::try_from_op semantics), host-only."""
    from mlxr_moe import _lib
    from mlxr_moe.moe import MoeConfig

    n = C.c_size_t(0)
    ok = MoeConfig(2048, 128, 8, 768).to_c()
    assert _lib.LIB.mlxr_cu_moe_workspace_size(C.byref(ok), 32, C.byref(n)) == 0
    assert n.value > 32 * 8 * 2048 * 2
    bad = MoeConfig(2048, 128, 8, 768, group_size=32).to_c()
    assert _lib.LIB.mlxr_cu_moe_workspace_size(C.byref(bad), 32, C.byref(n)) == _lib.ERR_UNSUPPORTED
    assert "group_size" in _lib.last_error()
    bad = MoeConfig(2000, 128, 8, 768).to_c()
    with pytest.raises(_lib.MlxrError) as ei:
        _lib.call("mlxr_cu_moe_workspace_size", C.byref(bad), 32, C.byref(n))
    assert ei.value.status == _lib.ERR_INVALID_ARGUMENT and "hidden_size" in ei.value.what
    bad = MoeConfig(2048, 128, 40, 768).to_c()
    assert _lib.LIB.mlxr_cu_moe_workspace_size(C.byref(bad), 32, C.byref(n)) == _lib.ERR_INVALID_ARGUMENT


def test_error_contract_op_family_args():
    from mlxr_moe import _lib

    assert _lib.LIB.mlxr_cu_quantize(None, 0, 4, 64, 64, 3, None, None, None, None, None) == _lib.ERR_UNSUPPORTED
    assert "bits=3" in _lib.last_error()
    assert _lib.LIB.mlxr_cu_quantize(None, 0, 4, 64, 64, 4, b"nvfp4", None, None, None, None) == _lib.ERR_UNSUPPORTED
    assert "nvfp4" in _lib.last_error()
    assert _lib.LIB.mlxr_cu_quantize(None, 0, 4, 100, 64, 4, None, None, None, None, None) == _lib.ERR_INVALID_ARGUMENT
    rc = _lib.LIB.mlxr_cu_gather_qmm(None, 0, 1, 1, 64, None, None, None, 1, 64, None, None, 1, 1, 64, 4, None, 0,
                                     None, None)
    assert rc == _lib.ERR_INVALID_ARGUMENT


def test_workspace_layout_grows_with_tokens():
    from mlxr_moe import _lib
    from mlxr_moe.moe import MoeConfig

    cfg = MoeConfig(2048, 512, 10, 512, shared_expert_intermediate_size=512, bits=8).to_c()
    sizes = []
    for T in (0, 1, 64, 4096, 16384):
        n = C.c_size_t(0)
        _lib.call("mlxr_cu_moe_workspace_size", C.byref(cfg), T, C.byref(n))
        sizes.append(n.value)
        assert n.value % 256 == 0
    assert sizes == sorted(sizes)


def test_host_index_broadcasting_matches_mlx_rules():
    """gather_qmm's absent indices are the arange over the batch, broadcast (quantization.rs:171)."""
    from mlxr_moe.ops import _broadcast_indices

    rhs = torch.tensor([[3, 1], [0, 2], [1, 1]], dtype=torch.int32)
    lf, rf, shape, nx, nw = _broadcast_indices(None, rhs, (3, 1), (4,), "cpu")
    assert shape == (3, 2) and nx == 3 and nw == 4
    assert lf.tolist() == [0, 0, 1, 1, 2, 2]
    assert rf.tolist() == [3, 1, 0, 2, 1, 1]
    lf, rf, shape, _, _ = _broadcast_indices(torch.tensor([0, 2]), torch.tensor([2, 1]), (5,), (3,), "cpu")
    assert shape == (2,) and lf.tolist() == [0, 2] and rf.tolist() == [2, 1]


def test_synth_stream_plan_and_work_model():
    from mlxr_moe import synth
    from mlxr_moe.moe import MoeConfig

    c = MoeConfig(2048, 128, 8, 768, bits=4)
    assert synth.expert_bytes(c) == 2654208  # 3*I*D*(b/8 + 4/64)
    assert synth.algorithmic_flops(c, 1) == 2 * 3 * 768 * 2048 * 8 + 2 * 128 * 2048
    c4 = synth.CONFIGS["c4"]["cfg"]
    assert synth.expert_bytes(c4) == 3342336
