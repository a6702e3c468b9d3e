"""Seeded synthetic blocks and inputs for the benchmark configurations.

There is no dataset on this path: the reference's block configurations are
defined by shapes and value distributions (weights N(0, 0.02) in bf16,
affine-quantised with group size 64; activations N(0, 1) in bf16). Values
come from Philox4x32-10 keyed by the seed with one counter stream per tensor
(router 0, switch gate 1, up 2, down 3, shared gate_proj 4, up_proj 5,
down_proj 6, shared_expert_gate 7, activations 8, expert ranking 9).
Generation and quantisation run on the GPU through the library.
"""
from __future__ import annotations

import math

import numpy as np
import torch

from . import ops
from .moe import (Gemma4MoeBranch, MoeConfig, PackedSwitchFfn, QuantizedLinear, QuantizedSwitchLinear, Qwen35MoeBlock,
                  SplitSwitchFfn, SwigluMlp)

STREAM_ROUTER, STREAM_GATE, STREAM_UP, STREAM_DOWN = 0, 1, 2, 3
STREAM_SH_GATE, STREAM_SH_UP, STREAM_SH_DOWN, STREAM_SH_EXPERT_GATE = 4, 5, 6, 7
STREAM_X, STREAM_RANK = 8, 9
STREAM_G4_ROUTER_NORM, STREAM_G4_EXPERT_SCALE, STREAM_G4_EXPERTS_NORM = 10, 11, 12

# BASELINE configurations (shapes only; the same block is reused across a
# config's token counts).
CONFIGS = {
    "c1": dict(cfg=MoeConfig(2048, 128, 8, 768, bits=4), tokens=[32], zipf=False),
    "c2": dict(cfg=MoeConfig(2048, 128, 8, 768, bits=4), tokens=[1, 8, 64], zipf=False),
    "c3": dict(cfg=MoeConfig(2048, 128, 8, 768, bits=4), tokens=[4096], zipf=True),
    "c4": dict(cfg=MoeConfig(2048, 512, 10, 512, shared_expert_intermediate_size=512, bits=8, shared_bits=8),
               tokens=[16384], zipf=False),
    "c5": dict(cfg=MoeConfig(4096, 128, 8, 1536, bits=4), tokens=[8192, 256], zipf=True),
}

# Zipf(1.1) routing skew: logit_bias[e] = -ZIPF_BETA * sigma * 1.1 * ln(rank(e)),
# sigma = 0.02 * sqrt(D), the standard deviation of a router logit for N(0, 0.02)
# router rows and N(0, 1) activations, so one beta gives the same skew at every
# hidden size. ZIPF_BETA = 0.62 minimises the L1 distance between the measured
# per-rank assignment shares and Zipf(1.1) capped at 1/K per expert (top-K
# without replacement, excess water-filled over the uncapped ranks), summed over
# 4096 C3-shaped and 8192 C5-shaped tokens (L1 0.217 and 0.222; top-1 share
# 0.099 against 0.125, top-8 0.452 against 0.510, ranks 65-128 0.085 against 0.112).
ZIPF_S = 1.1
ZIPF_BETA = 0.62


def expert_ranks(num_experts: int, seed: int = 0, device="cuda") -> np.ndarray:
    """A seeded permutation of 1..E (rank of each expert)."""
    keys = ops.synth_normal_bf16(seed, STREAM_RANK, (num_experts,), 1.0, device).float().cpu().numpy()
    order = np.argsort(keys, kind="stable")
    ranks = np.empty(num_experts, np.int64)
    ranks[order] = np.arange(1, num_experts + 1)
    return ranks


def router_logit_sigma(hidden: int) -> float:
    return 0.02 * math.sqrt(hidden)


def zipf_bias(num_experts: int, hidden: int, seed: int = 0, beta: float = ZIPF_BETA, s: float = ZIPF_S,
              device="cuda"):
    r = expert_ranks(num_experts, seed, device)
    scale = beta * router_logit_sigma(hidden) * s
    return torch.tensor(-scale * np.log(r.astype(np.float64)), dtype=torch.float32, device=device)


def _qswitch(seed, stream, shape, cfg_bits, gs, device):
    w = ops.synth_normal_bf16(seed, stream, shape, 0.02, device)
    q = QuantizedSwitchLinear.from_switch_linear(w, gs, cfg_bits)
    del w
    return q


def make_block(cfg: MoeConfig, seed: int = 0, zipf: bool = False, device="cuda") -> Qwen35MoeBlock:
    D, E, I, Is = cfg.hidden_size, cfg.num_experts, cfg.moe_intermediate_size, cfg.shared_expert_intermediate_size
    gs, b = cfg.group_size, cfg.bits
    sb = cfg.shared_bits if cfg.shared_bits is not None else b
    router = ops.synth_normal_bf16(seed, STREAM_ROUTER, (E, D), 0.02, device)
    sw = SplitSwitchFfn(
        _qswitch(seed, STREAM_GATE, (E, I, D), b, gs, device),
        _qswitch(seed, STREAM_UP, (E, I, D), b, gs, device),
        _qswitch(seed, STREAM_DOWN, (E, D, I), b, gs, device),
    )
    shared = shared_gate = None
    if Is > 0:
        def ql(stream, shape):
            w = ops.synth_normal_bf16(seed, stream, shape, 0.02, device)
            return QuantizedLinear.from_linear(w, gs, sb)

        shared = SwigluMlp(ql(STREAM_SH_GATE, (Is, D)), ql(STREAM_SH_UP, (Is, D)), ql(STREAM_SH_DOWN, (D, Is)))
        shared_gate = ql(STREAM_SH_EXPERT_GATE, (1, D))
    bias = zipf_bias(E, D, seed, device=device) if zipf else None
    return Qwen35MoeBlock(cfg, router, sw, shared, shared_gate, bias)


def make_input(num_tokens: int, hidden: int, seed: int = 0, stream_offset: int = 0, device="cuda") -> torch.Tensor:
    """x [T, D] bf16 N(0, 1); stream_offset separates batches of one config."""
    return ops.synth_normal_bf16(seed, STREAM_X + 16 * stream_offset, (num_tokens, hidden), 1.0, device)


def expert_bytes(cfg: MoeConfig) -> int:
    """B_e = 3 * I * D * (bits/8 + 4/64): packed codes + bf16 scale and bias per 64."""
    return int(3 * cfg.moe_intermediate_size * cfg.hidden_size * (cfg.bits / 8 + 4 / 64))


def algorithmic_bytes(cfg: MoeConfig, num_tokens: int, distinct_experts: int) -> int:
    """U*B_e + router + shared expert + x in + out."""
    D, E = cfg.hidden_size, cfg.num_experts
    byts = distinct_experts * expert_bytes(cfg) + E * D * 2 + 2 * num_tokens * D * 2
    Is = cfg.shared_expert_intermediate_size
    if Is:
        sb = cfg.shared_bits if cfg.shared_bits is not None else cfg.bits
        byts += int((3 * Is * D + D) * (sb / 8 + 4 / 64))
    return byts


def algorithmic_flops(cfg: MoeConfig, num_tokens: int) -> int:
    """2*3*I*D*K + 2*E*D per token (+ 2*3*Is*D + 2*D with a shared expert)."""
    D, E, K, I, Is = (cfg.hidden_size, cfg.num_experts, cfg.num_experts_per_tok, cfg.moe_intermediate_size,
                      cfg.shared_expert_intermediate_size)
    f = 2 * 3 * I * D * K + 2 * E * D
    if Is:
        f += 2 * 3 * Is * D + 2 * D
    return num_tokens * f


def make_gemma4_branch(cfg: MoeConfig, seed: int = 0, device="cuda") -> Gemma4MoeBranch:
    """A seeded Gemma 4 MoE branch (no checkpoint is available here): router
    proj N(0, 0.5) bf16 (scores of order one on the RMS-normed input),
    router_norm = bf16(hidden^-0.5 * (1 + N(0, 0.1))), per_expert_scale
    1 + N(0, 0.2), experts_norm 1 + N(0, 0.1), gate_up_proj [E, 2I, D] and
    down_proj [E, D, I] N(0, 0.02) affine-quantised. Streams: router 0,
    gate_up 1, down 3, the three norm/scale vectors 10-12."""
    D, E, I = cfg.hidden_size, cfg.num_experts, cfg.moe_intermediate_size
    gs, b = cfg.group_size, cfg.bits
    proj = ops.synth_normal_bf16(seed, STREAM_ROUTER, (E, D), 0.5, device)

    def around_one(stream, n, sd):
        return (1.0 + ops.synth_normal_bf16(seed, stream, (n,), sd, device).float()).to(torch.bfloat16)

    router_norm = (around_one(STREAM_G4_ROUTER_NORM, D, 0.1).float() * D ** -0.5).to(torch.bfloat16)
    ffn = PackedSwitchFfn(_qswitch(seed, STREAM_GATE, (E, 2 * I, D), b, gs, device),
                          _qswitch(seed, STREAM_DOWN, (E, D, I), b, gs, device))
    return Gemma4MoeBranch(cfg, proj, router_norm, around_one(STREAM_G4_EXPERT_SCALE, E, 0.2),
                           around_one(STREAM_G4_EXPERTS_NORM, D, 0.1), ffn)
