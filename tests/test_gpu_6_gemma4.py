"""The Gemma 4 MoE branch (model_kind 1: RMS-normed router with
router_post, experts on pre_feedforward_layernorm_2(h) through a packed
gate_up_proj with GeGLU) on the GPU against the oracle: routing bit-exact,
outputs within the block tolerance. T = 1 and 16 take the split router and
the split-K / fused decode GEMMs, 100 the one-CTA router, 300 the tiled
logits kernel and wide tiles."""
import numpy as np
import pytest
import torch

import oracle as O
from conftest import ATOL, RTOL, assert_close_bf16, bf16_np
from gpu_helpers import qtriple, run_gpu_block
from mlxr_moe import MlxrError, synth
from mlxr_moe.moe import MoeConfig

pytestmark = pytest.mark.gpu

CFG = MoeConfig(1024, 64, 4, 512, bits=4, model_kind=1, rms_norm_eps=1e-6)


@pytest.fixture(scope="module")
def branch():
    return synth.make_gemma4_branch(CFG, 0)


def oracle_weights(b):
    u16 = lambda t: t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    return {
        "router": u16(b.gate), "router_norm": u16(b.router_norm), "expert_scale": u16(b.expert_scale),
        "experts_norm": u16(b.experts_norm), "gate_up": qtriple(b.switch_glu.gate_up_proj),
        "down": qtriple(b.switch_glu.down_proj),
    }


def oracle_cfg(c):
    return dict(hidden=c.hidden_size, num_experts=c.num_experts, top_k=c.num_experts_per_tok,
                moe_intermediate=c.moe_intermediate_size, group_size=c.group_size, bits=c.bits, eps=c.rms_norm_eps)


@pytest.mark.parametrize("T", [1, 16, 100, 300])
def test_gemma4_branch_matches_oracle(branch, T):
    x = synth.make_input(T, CFG.hidden_size, 0, 40 + T)
    out, r = run_gpu_block(branch, x)
    o, idx, w = O.gemma4_block(oracle_cfg(CFG), oracle_weights(branch), bf16_np(x))
    np.testing.assert_array_equal(r.indices.cpu().numpy(), idx)
    np.testing.assert_array_equal(bf16_np(r.weights), w)
    assert_close_bf16(bf16_np(out), o, ATOL, RTOL, "gemma4 branch vs oracle")


def test_gemma4_router_substep(branch):
    x = synth.make_input(40, CFG.hidden_size, 0, 90)
    idx, w = branch.router(x)
    torch.cuda.synchronize()
    _, oidx, ow = O.gemma4_block(oracle_cfg(CFG), oracle_weights(branch), bf16_np(x), routing_only=True)
    np.testing.assert_array_equal(idx.cpu().numpy(), oidx)
    np.testing.assert_array_equal(bf16_np(w), ow)


def test_gemma4_rejects_shared_expert_and_bad_kind():
    bad = MoeConfig(1024, 64, 4, 512, shared_expert_intermediate_size=512, model_kind=1)
    with pytest.raises(ValueError):
        synth.make_gemma4_branch(bad, 0)
    from mlxr_moe import _lib
    import ctypes as C
    c = MoeConfig(1024, 64, 4, 512, model_kind=7).to_c()
    n = C.c_size_t(0)
    with pytest.raises(MlxrError):
        _lib.call("mlxr_cu_moe_workspace_size", C.byref(c), 16, C.byref(n))
