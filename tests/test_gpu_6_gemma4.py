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


# ----------------------------------------------------- checkpoint ingest ----
def _ckpt_tensors(prefix, split_quantised, seed=3):
    """Tensors of one Gemma 4 MoE layer as a checkpoint stores them, and the
    oracle's view of the same weights (device-quantised on the GPU)."""
    from mlxr_moe import ops
    D, E, K, I = CFG.hidden_size, CFG.num_experts, CFG.num_experts_per_tok, CFG.moe_intermediate_size
    u16 = lambda t: t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    g = lambda st, shape, sd: ops.synth_normal_bf16(seed, st, shape, sd, "cuda")  # noqa: E731
    proj = g(0, (E, D), 0.5)
    scale = (1.0 + g(10, (D,), 0.1).float()).to(torch.bfloat16)
    pes = (1.0 + g(11, (E,), 0.2).float()).to(torch.bfloat16)
    pre2 = (1.0 + g(12, (D,), 0.1).float()).to(torch.bfloat16)
    gate, up, down = g(1, (E, I, D), 0.02), g(2, (E, I, D), 0.02), g(3, (E, D, I), 0.02)
    T = {f"{prefix}.router.proj.weight": u16(proj), f"{prefix}.router.scale": u16(scale),
         f"{prefix}.router.per_expert_scale": u16(pes), f"{prefix}.pre_feedforward_layernorm_2.weight": u16(pre2)}
    q3 = lambda w: tuple(x.cpu().numpy().view(np.uint32) if i == 0 else u16(x)  # noqa: E731
                         for i, x in enumerate(ops.quantize(w, 64, 4)))
    if split_quantised:
        for name, w in (("gate_proj", gate), ("up_proj", up), ("down_proj", down)):
            for part, a in zip(("weight", "scales", "biases"), q3(w)):
                T[f"{prefix}.experts.{name}.{part}"] = a
        qg, qu, qd = (tuple(T[f"{prefix}.experts.{n}.{p}"] for p in ("weight", "scales", "biases"))
                      for n in ("gate_proj", "up_proj", "down_proj"))
        gate_up = tuple(np.concatenate([a, b], axis=1) for a, b in zip(qg, qu))
    else:
        T[f"{prefix}.experts.gate_up_proj"] = u16(torch.cat([gate, up], 1))
        T[f"{prefix}.experts.down_proj"] = u16(down)
        gate_up = qd = None  # quantised by the loader; read back from the branch
    root = np.float32(D ** -0.5)
    rn = O.f32_to_bf16(O.bf16_to_f32(T[f"{prefix}.router.scale"]) * O.bf16_to_f32(O.f32_to_bf16(root)))
    W = {"router": T[f"{prefix}.router.proj.weight"], "router_norm": rn,
         "expert_scale": T[f"{prefix}.router.per_expert_scale"],
         "experts_norm": T[f"{prefix}.pre_feedforward_layernorm_2.weight"], "gate_up": gate_up, "down": qd}
    return T, W


@pytest.mark.parametrize("split_quantised", [True, False])
def test_gemma4_checkpoint_branch(tmp_path, split_quantised):
    import json

    from mlxr_moe import checkpoint as ck
    prefix = "model.language_model.layers.2"
    T, W = _ckpt_tensors(prefix, split_quantised)
    ck.write_safetensors(str(tmp_path / "model.safetensors"), T)
    with open(tmp_path / "config.json", "w") as f:
        json.dump({"text_config": {"hidden_size": CFG.hidden_size, "num_experts": CFG.num_experts,
                                   "top_k_experts": CFG.num_experts_per_tok,
                                   "moe_intermediate_size": CFG.moe_intermediate_size, "rms_norm_eps": 1e-6},
                   "quantization": {"group_size": 64, "bits": 4}}, f)
    b = ck.load_gemma4_moe_branch(str(tmp_path), 2)
    np.testing.assert_array_equal(bf16_np(b.router_norm), W["router_norm"])
    if not split_quantised:  # the loader quantised the dense experts on the device
        W["gate_up"], W["down"] = qtriple(b.switch_glu.gate_up_proj), qtriple(b.switch_glu.down_proj)
    else:
        np.testing.assert_array_equal(qtriple(b.switch_glu.gate_up_proj)[0], W["gate_up"][0])
    x = synth.make_input(40, CFG.hidden_size, 0, 95)
    out, r = run_gpu_block(b, x)
    o, idx, w = O.gemma4_block(oracle_cfg(CFG), W, bf16_np(x))
    np.testing.assert_array_equal(r.indices.cpu().numpy(), idx)
    np.testing.assert_array_equal(bf16_np(r.weights), w)
    assert_close_bf16(bf16_np(out), o, ATOL, RTOL, "gemma4 checkpoint branch vs oracle")
