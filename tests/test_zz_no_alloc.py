"""The allocation-free block entry point, for callers that cannot allocate
device memory when they call the library (an engine that has reserved the
GPU's memory up front, or a runtime that binds the C ABI without a device
allocator). It must give the same result as the workspace entry point, on
consecutive calls that share its built-in scratch.

Collected last on purpose: if it fails, a run that stops at the first failure
has already run every other test."""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle as O
from conftest import ATOL, RTOL, assert_close_bf16, bf16_np
from gpu_helpers import block_to_oracle

pytestmark = pytest.mark.gpu


def _noalloc(blk, x, out, status):
    from mlxr_moe import _lib

    st = torch.cuda.current_stream().cuda_stream
    return _lib.LIB.mlxr_cu_moe_block_forward_noalloc(C.byref(blk._ccfg), C.byref(blk._cw), x.data_ptr(),
                                                      x.shape[0], out.data_ptr(), None, status.data_ptr(), st)


def test_noalloc_matches_workspace_entry_point_on_consecutive_calls():
    from mlxr_moe import _lib, synth

    blk = synth.make_block(synth.CONFIGS["c2"]["cfg"], seed=0)
    cfg, W = block_to_oracle(blk)
    status = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    for call, (T, offset) in enumerate(((64, 31), (8, 32))):  # two calls in a row, different inputs
        x = synth.make_input(T, 2048, stream_offset=offset)
        want = blk.forward(x)
        got = torch.empty_like(x)
        rc = _noalloc(blk, x, got, status)
        assert rc == _lib.OK, _lib.last_error()
        torch.cuda.synchronize()
        assert int(status.item()) == 0, f"device status {int(status.item())} on call {call}"
        assert_close_bf16(bf16_np(got), bf16_np(want), ATOL, RTOL, f"noalloc call {call}")
        # and directly against the CPU oracle on the same inputs
        o_fu, _, _ = O.moe_block(cfg, W, bf16_np(x), "fused")
        assert_close_bf16(bf16_np(got), o_fu, ATOL, RTOL, f"noalloc call {call} vs oracle")


def test_noalloc_rejects_batches_beyond_its_scratch():
    from mlxr_moe import _lib, synth

    blk = synth.make_block(synth.CONFIGS["c2"]["cfg"], seed=0)
    x = torch.zeros((4096, 2048), dtype=torch.bfloat16, device="cuda")
    out = torch.empty_like(x)
    status = torch.zeros((1,), dtype=torch.int32, device="cuda")
    rc = _noalloc(blk, x, out, status)
    assert rc == _lib.ERR_WORKSPACE
    assert "allocation-free" in _lib.last_error()
    _lib.LIB.mlxr_cu_clear_error()
    np.testing.assert_array_equal(status.cpu().numpy(), [0])
