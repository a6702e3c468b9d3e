"""A converted checkpoint (the mlxr-convert layout: sharded safetensors +
index, 4-bit experts and shared expert, 8-bit router and shared-expert gate)
loaded with load_qwen35_moe_block at the Qwen3.6-35B-A3B block shape
(D=2048, E=256, K=8, I=Is=512), run on the GPU, against the oracle."""
import json

import numpy as np
import pytest
import torch

import oracle as O
from conftest import ATOL, RTOL, assert_close_bf16, bf16_np
from gpu_helpers import run_gpu_block
from mlxr_moe import checkpoint as ck
from mlxr_moe import ops

pytestmark = pytest.mark.gpu

D, E, K, I, IS = 2048, 256, 8, 512, 512
LAYER = 3


def _quant(seed, stream, shape, bits):
    w = ops.synth_normal_bf16(seed, stream, shape, 0.02, "cuda")
    wq, s, b = ops.quantize(w, 64, bits)
    return (wq.cpu().numpy().view(np.uint32), s.cpu().view(torch.int16).numpy().view(np.uint16),
            b.cpu().view(torch.int16).numpy().view(np.uint16))


@pytest.fixture(scope="module")
def converted(tmp_path_factory):
    d = tmp_path_factory.mktemp("a3b_like")
    p = ck.layer_prefix(LAYER)
    W = {"router_q": _quant(0, 0, (E, D), 8), "gate": _quant(0, 1, (E, I, D), 4), "up": _quant(0, 2, (E, I, D), 4),
         "down": _quant(0, 3, (E, D, I), 4), "sh_gate": _quant(0, 4, (IS, D), 4), "sh_up": _quant(0, 5, (IS, D), 4),
         "sh_down": _quant(0, 6, (D, IS), 4), "sh_expert_gate": _quant(0, 7, (1, D), 8)}
    names = {"router_q": "gate", "gate": "switch_mlp.gate_proj", "up": "switch_mlp.up_proj",
             "down": "switch_mlp.down_proj", "sh_gate": "shared_expert.gate_proj",
             "sh_up": "shared_expert.up_proj", "sh_down": "shared_expert.down_proj",
             "sh_expert_gate": "shared_expert_gate"}
    shards = [{}, {}]
    for i, (k, n) in enumerate(names.items()):
        for part, arr in zip(("weight", "scales", "biases"), W[k]):
            shards[i % 2][f"{p}.{n}.{part}"] = arr
    wmap = {}
    for i, sh in enumerate(shards):
        fn = f"model-{i + 1:05d}-of-00002.safetensors"
        ck.write_safetensors(str(d / fn), sh)
        wmap.update({k: fn for k in sh})
    with open(d / "model.safetensors.index.json", "w") as f:
        json.dump({"metadata": {"total_size": 0}, "weight_map": wmap}, f)
    q = {"group_size": 64, "bits": 4, "mode": "affine", f"{p}.gate": {"group_size": 64, "bits": 8},
         f"{p}.shared_expert_gate": {"group_size": 64, "bits": 8}}
    with open(d / "config.json", "w") as f:
        json.dump({"text_config": {"hidden_size": D, "num_experts": E, "num_experts_per_tok": K,
                                   "moe_intermediate_size": I, "shared_expert_intermediate_size": IS},
                   "quantization": q}, f)
    return str(d), W


def _oracle(W, x):
    cfg = dict(hidden=D, num_experts=E, top_k=K, moe_intermediate=I, shared_intermediate=IS, group_size=64, bits=4,
               shared_bits=4, shared_gate_bits=8)
    Wo = dict(W)
    Wo["router"] = O.dequantize(*W["router_q"], 64, 8, out_dtype=np.uint16)  # bf16(scale * q + bias)
    del Wo["router_q"]
    return O.moe_block(cfg, Wo, x, "fused")


@pytest.mark.parametrize("T", [16, 300])
def test_converted_checkpoint_block(converted, T):
    path, W = converted
    blk = ck.load_qwen35_moe_block(path, LAYER)
    c = blk.cfg
    assert (c.num_experts, c.bits, c.shared_bits, c.shared_gate_bits) == (E, 4, 4, 8)
    x = ops.synth_normal_bf16(0, 8 + 16 * T, (T, D), 1.0, "cuda")
    out, r = run_gpu_block(blk, x)
    o, idx, w = _oracle(W, bf16_np(x))
    np.testing.assert_array_equal(r.indices.cpu().numpy(), idx)
    np.testing.assert_array_equal(bf16_np(r.weights), w)
    assert_close_bf16(bf16_np(out), o, ATOL, RTOL, "converted checkpoint vs oracle")


def test_loader_rejects_mismatched_shapes(converted, tmp_path):
    path, _ = converted
    cfgj = json.load(open(f"{path}/config.json"))
    cfgj["text_config"]["moe_intermediate_size"] = 256  # the stored experts have I = 512
    m = ck.Checkpoint(path)
    m.config = cfgj
    with pytest.raises(ValueError):
        ck.load_qwen35_moe_block(m, LAYER)
