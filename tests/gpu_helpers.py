"""Helpers shared by the GPU parity tests: move a device block to the oracle's
host representation and run both sides on the same inputs."""
import numpy as np
import torch

import oracle as O
from conftest import bf16_np


def u32(t):
    return t.detach().contiguous().cpu().numpy().view(np.uint32)


def qtriple(q):
    return (u32(q.weight), bf16_np(q.scales), bf16_np(q.biases))


def block_to_oracle(block):
    c = block.cfg
    cfg = dict(hidden=c.hidden_size, num_experts=c.num_experts, top_k=c.num_experts_per_tok,
               moe_intermediate=c.moe_intermediate_size, shared_intermediate=c.shared_expert_intermediate_size,
               group_size=c.group_size, bits=c.bits, shared_bits=c.shared_bits if c.shared_bits else c.bits,
               renorm=c.norm_topk_prob, shared_gate_bits=c.shared_gate_bits or 0)
    sm = block.switch_mlp
    W = {"router": bf16_np(block.gate), "gate": qtriple(sm.gate_proj), "up": qtriple(sm.up_proj),
         "down": qtriple(sm.down_proj)}
    if block.router_bias is not None:
        W["router_bias"] = block.router_bias.cpu().numpy().astype(np.float32)
    if block.shared_expert is not None:
        se = block.shared_expert
        W["sh_gate"] = qtriple(se.gate_proj)
        W["sh_up"] = qtriple(se.up_proj)
        W["sh_down"] = qtriple(se.down_proj)
        W["sh_expert_gate"] = qtriple(block.shared_expert_gate)
    return cfg, W


def run_gpu_block(block, x):
    from mlxr_moe.moe import Routing

    T = x.shape[0]
    r = Routing(T, block.cfg.num_experts_per_tok, block.cfg.num_experts, x.device)
    out = block.forward(x, routing=r)
    block.status()
    torch.cuda.synchronize()
    return out, r
