"""Regenerates the committed golden fixtures from the CPU oracle.

Run from the repo root: `python tests/golden/make_golden.py`. The fixtures
pin the oracle's routing contract, packing and both block modes on small
blocks (D=256, E=16, K=4, I=128, 4-bit gs64; an 8-bit block with a shared
expert; a skewed-router block) so that any change to the oracle is visible,
and give the GPU tests fixed inputs with known outputs. Weights are not
stored: they are regenerated from the seeded generator by `small_block` and
pinned by SHA-256 digests. `gemma4_small.npz` pins the Gemma 4 branch
(orc_gemma4_block) the same way.
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
import oracle as O  # noqa: E402


def small_block(seed, D, E, K, I, T, bits, Is=0, zipf=False):
    W = {"router": O.normal_bf16(seed, 0, (E, D), 0.02)}
    W["gate"] = O.quantize(O.normal_bf16(seed, 1, (E, I, D), 0.02), 64, bits)
    W["up"] = O.quantize(O.normal_bf16(seed, 2, (E, I, D), 0.02), 64, bits)
    W["down"] = O.quantize(O.normal_bf16(seed, 3, (E, D, I), 0.02), 64, bits)
    if Is:
        W["sh_gate"] = O.quantize(O.normal_bf16(seed, 4, (Is, D), 0.02), 64, bits)
        W["sh_up"] = O.quantize(O.normal_bf16(seed, 5, (Is, D), 0.02), 64, bits)
        W["sh_down"] = O.quantize(O.normal_bf16(seed, 6, (D, Is), 0.02), 64, bits)
        W["sh_expert_gate"] = O.quantize(O.normal_bf16(seed, 7, (1, D), 0.02), 64, bits)
    if zipf:
        W["router_bias"] = (-1.1 * np.log(np.arange(1, E + 1, dtype=np.float64)[::-1])).astype(np.float32)
    x = O.normal_bf16(seed, 8, (T, D), 1.0)
    cfg = dict(hidden=D, num_experts=E, top_k=K, moe_intermediate=I, shared_intermediate=Is, group_size=64,
               bits=bits, shared_bits=bits)
    return cfg, W, x


def small_gemma4(seed, D, E, K, I, T, bits=4):
    """A small Gemma 4 MoE branch (the oracle's orc_gemma4_block inputs)."""
    f = lambda a: O.bf16_to_f32(a)  # noqa: E731
    W = {"router": O.normal_bf16(seed, 0, (E, D), 0.5),
         "router_norm": O.f32_to_bf16(np.float32(D ** -0.5) * (1.0 + f(O.normal_bf16(seed, 10, (D,), 0.1)))),
         "expert_scale": O.f32_to_bf16(1.0 + f(O.normal_bf16(seed, 11, (E,), 0.2))),
         "experts_norm": O.f32_to_bf16(1.0 + f(O.normal_bf16(seed, 12, (D,), 0.1))),
         "gate_up": O.quantize(O.normal_bf16(seed, 1, (E, 2 * I, D), 0.02), 64, bits),
         "down": O.quantize(O.normal_bf16(seed, 3, (E, D, I), 0.02), 64, bits)}
    x = O.normal_bf16(seed, 8, (T, D), 1.0)
    cfg = dict(hidden=D, num_experts=E, top_k=K, moe_intermediate=I, group_size=64, bits=bits, eps=1e-6)
    return cfg, W, x


GEMMA4 = {"g4": dict(seed=0, D=256, E=16, K=4, I=128, T=12)}

BLOCKS = {
    "q4": dict(seed=0, D=256, E=16, K=4, I=128, T=10, bits=4),
    "q8s": dict(seed=1, D=256, E=16, K=4, I=128, T=7, bits=8, Is=128),
    "q4z": dict(seed=2, D=256, E=16, K=4, I=128, T=33, bits=4, zipf=True),
}


def digest(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def flat(prefix, W):
    out = {}
    for k, v in W.items():
        if isinstance(v, tuple):
            out[f"{prefix}{k}.weight"], out[f"{prefix}{k}.scales"], out[f"{prefix}{k}.biases"] = v
        else:
            out[f"{prefix}{k}"] = v
    return out


def main():
    fx = {}
    for name, args in BLOCKS.items():
        cfg, W, x = small_block(**args)
        o_st, idx, w = O.moe_block(cfg, W, x, "staged")
        o_fu, idx2, w2 = O.moe_block(cfg, W, x, "fused")
        assert (idx == idx2).all() and (w == w2).all()
        _, _, lg, pr = O.router(x, W["router"], cfg["top_k"], W.get("router_bias"), True, want_logits=True)
        for k, v in flat(f"{name}/", W).items():
            fx[k + ".sha256"] = np.array(digest(v))
        fx[f"{name}/x"] = x
        fx[f"{name}/cfg"] = np.array([cfg[k] for k in ("hidden", "num_experts", "top_k", "moe_intermediate",
                                                       "shared_intermediate", "group_size", "bits", "shared_bits")])
        fx[f"{name}/out_staged"] = o_st
        fx[f"{name}/out_fused"] = o_fu
        fx[f"{name}/idx"] = idx
        fx[f"{name}/w"] = w
        fx[f"{name}/logits"] = lg
        fx[f"{name}/probs"] = pr
    # quantiser on the reference's own test matrix (quantization.rs:299-315).
    xx = (np.ones((128, 1), np.float32) * np.arange(512, dtype=np.float32)[None, :]).astype(np.float32)
    for b in (2, 4, 8):
        q, s, bb = O.quantize(xx, 128, b)
        fx[f"quant_arange/b{b}.weight"], fx[f"quant_arange/b{b}.scales"], fx[f"quant_arange/b{b}.biases"] = q, s, bb
    # the generator itself: first values of a few streams.
    for st in (0, 1, 8):
        fx[f"normal/seed0_stream{st}"] = O.normal_bf16(0, st, (4096,), 1.0)
    np.savez_compressed(os.path.join(HERE, "moe_small.npz"), **fx)
    print("wrote", os.path.join(HERE, "moe_small.npz"), len(fx), "arrays")
    # The Gemma 4 branch (orc_gemma4_block) in its own file.
    gx = {}
    for name, args in GEMMA4.items():
        cfg, W, x = small_gemma4(**args)
        out, idx, w = O.gemma4_block(cfg, W, x)
        for k, v in flat(f"{name}/", W).items():
            gx[k + ".sha256"] = np.array(digest(v))
        gx[f"{name}/x"], gx[f"{name}/out"], gx[f"{name}/idx"], gx[f"{name}/w"] = x, out, idx, w
    np.savez_compressed(os.path.join(HERE, "gemma4_small.npz"), **gx)
    print("wrote", os.path.join(HERE, "gemma4_small.npz"), len(gx), "arrays")


if __name__ == "__main__":
    main()
