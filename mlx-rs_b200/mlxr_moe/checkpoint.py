"""Qwen 3.5 / 3.6 MoE blocks (and the Gemma 4 MoE branch, see below) from
a converted checkpoint directory.

The converter (crates/mlxr-convert) writes:
  * sharded safetensors files plus `model.safetensors.index.json`, whose
    `weight_map` names the shard of every tensor (shards.rs:24-117); a
    single `model.safetensors` is accepted too;
  * every quantised tensor as `{stem}.weight` (packed uint32), `{stem}.scales`
    and `{stem}.biases` (quantize.rs:22-58);
  * the experts, after splitting the source's packed `gate_up_proj`, under
    `language_model.model.layers.N.mlp.switch_mlp.{gate,up,down}_proj`
    (qwen3_5.rs:96-150), the router at `...mlp.gate` and the shared expert
    at `...mlp.shared_expert.{gate,up,down}_proj` and
    `...mlp.shared_expert_gate`, the last two pinned at 8 bits, group 64
    (qwen3_5.rs, classify_default).
`config.json` carries the model dimensions (under `text_config` for the
vision-language release) and the quantisation block with per-path overrides,
read as QuantizationConfig.for_path does (crates/mlxr-lm/src/quantization.rs).

The block's router reads bf16 rows; a quantised router is expanded once, at
load, to bf16(scale * q + bias) with the library's dequantize (the values the
op family's quantized_matmul multiplies by).
"""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass, field

import numpy as np
import torch

from . import ops
from .moe import (Gemma4MoeBranch, MoeConfig, PackedSwitchFfn, QuantizedLinear, QuantizedSwitchLinear, Qwen35MoeBlock,
                  SplitSwitchFfn, SwigluMlp)

# ------------------------------------------------------------ config -----


@dataclass
class QuantizationConfig:
    """config.json `quantization` (crates/mlxr-lm/src/quantization.rs:18-66):
    global group size and bits, mode "affine", and per-path overrides given
    as `{"<prefix>": {"group_size": g, "bits": b}}` entries."""

    group_size: int
    bits: int
    mode: str = "affine"
    overrides: dict = field(default_factory=dict)

    @classmethod
    def from_dict(cls, d: dict) -> "QuantizationConfig":
        if "group_size" not in d or "bits" not in d:
            raise ValueError("quantization config needs group_size and bits")
        mode = d.get("mode", "affine")
        if mode != "affine":
            raise ValueError(f"quantization mode {mode!r} is not supported (affine)")
        ov = {}
        for k, v in d.items():
            if isinstance(v, dict) and "group_size" in v and "bits" in v:
                ov[k] = (int(v["group_size"]), int(v["bits"]))
        return cls(int(d["group_size"]), int(d["bits"]), mode, ov)

    def for_path(self, raw_prefix: str) -> tuple[int, int]:
        """(group_size, bits) of the tensor at `raw_prefix` (no `.weight`)."""
        return self.overrides.get(raw_prefix, (self.group_size, self.bits))


def text_config(config: dict) -> dict:
    """The decoder's fields: `text_config` of a VLM-style config, else the config itself."""
    return config.get("text_config", config)


def quantization_config(config: dict) -> QuantizationConfig | None:
    q = config.get("quantization", config.get("quantization_config"))
    return None if q is None else QuantizationConfig.from_dict(q)


def layer_prefix(layer: int) -> str:
    return f"language_model.model.layers.{layer}.mlp"


def moe_config(config: dict, layer: int = 0) -> MoeConfig:
    """MoeConfig of one layer's block from config.json (config.rs field names;
    bit widths from the quantisation block's overrides for that layer)."""
    tc = text_config(config)
    q = quantization_config(config)
    if q is None:
        raise ValueError("the block needs quantised experts: config.json has no quantization block")
    p = layer_prefix(layer)
    gs, bits = q.for_path(f"{p}.switch_mlp.gate_proj")
    Is = int(tc.get("shared_expert_intermediate_size", 0) or 0)
    sgs, sbits = q.for_path(f"{p}.shared_expert.gate_proj")
    ggs, gbits = q.for_path(f"{p}.shared_expert_gate")
    for name, g in (("experts", gs), ("shared expert", sgs), ("shared expert gate", ggs)):
        if g != 64:
            raise ValueError(f"{name}: group size {g} is not supported by the block (64)")
    return MoeConfig(
        hidden_size=int(tc["hidden_size"]), num_experts=int(tc["num_experts"]),
        num_experts_per_tok=int(tc["num_experts_per_tok"]), moe_intermediate_size=int(tc["moe_intermediate_size"]),
        shared_expert_intermediate_size=Is, group_size=gs, bits=bits, shared_bits=sbits if Is else None,
        norm_topk_prob=bool(tc.get("norm_topk_prob", True)), shared_gate_bits=gbits if Is else None,
    )


# ------------------------------------------------------- safetensors -----

_DTYPES = {"U32": np.uint32, "I32": np.int32, "BF16": np.uint16, "F16": np.float16, "F32": np.float32,
           "U8": np.uint8, "I64": np.int64}


def read_header(path: str) -> tuple[dict, int]:
    """(tensor entries, byte offset of the data section) of a safetensors file."""
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(n))
    header.pop("__metadata__", None)
    return header, 8 + n


def write_safetensors(path: str, tensors: dict, dtypes: dict | None = None) -> None:
    """Write numpy arrays as one safetensors file (the converter's on-disk
    format). `dtypes` names the stored dtype per key; uint16 arrays default to
    BF16 (bf16 bit patterns)."""
    dtypes = dtypes or {}
    rev = {np.dtype(v): k for k, v in _DTYPES.items()}
    header, off, blobs = {}, 0, []
    for k in sorted(tensors):
        a = np.ascontiguousarray(tensors[k])
        dt = dtypes.get(k) or rev[a.dtype]
        b = a.tobytes()
        header[k] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        off += len(b)
        blobs.append(b)
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


class Checkpoint:
    """Tensors of a converted model directory, read on demand."""

    def __init__(self, model_dir: str):
        self.dir = model_dir
        idx = os.path.join(model_dir, "model.safetensors.index.json")
        if os.path.exists(idx):
            with open(idx) as f:
                self.weight_map = json.load(f)["weight_map"]
        else:
            single = os.path.join(model_dir, "model.safetensors")
            if not os.path.exists(single):
                raise FileNotFoundError(f"{model_dir}: no model.safetensors.index.json or model.safetensors")
            self.weight_map = {k: "model.safetensors" for k in read_header(single)[0]}
        self._headers = {}
        with open(os.path.join(model_dir, "config.json")) as f:
            self.config = json.load(f)

    def __contains__(self, key: str) -> bool:
        return key in self.weight_map

    def numpy(self, key: str) -> np.ndarray:
        if key not in self.weight_map:
            raise KeyError(f"{key} is not in the checkpoint")
        shard = os.path.join(self.dir, self.weight_map[key])
        if shard not in self._headers:
            self._headers[shard] = read_header(shard)
        header, base = self._headers[shard]
        e = header[key]
        if e["dtype"] not in _DTYPES:
            raise ValueError(f"{key}: dtype {e['dtype']} is not supported")
        lo, hi = e["data_offsets"]
        with open(shard, "rb") as f:
            f.seek(base + lo)
            buf = f.read(hi - lo)
        return np.frombuffer(buf, dtype=_DTYPES[e["dtype"]]).reshape(e["shape"])

    def tensor(self, key: str, device) -> torch.Tensor:
        """Device tensor: packed uint32 as int32 bit patterns, BF16 as bfloat16, others as is."""
        a = self.numpy(key)
        if a.dtype == np.uint32:
            return torch.from_numpy(a.view(np.int32).copy()).to(device)
        if a.dtype == np.uint16:
            return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).to(device)
        return torch.from_numpy(a.copy()).to(device)

    def dtype_of(self, key: str) -> str:
        shard = os.path.join(self.dir, self.weight_map[key])
        if shard not in self._headers:
            self._headers[shard] = read_header(shard)
        return self._headers[shard][0][key]["dtype"]


# --------------------------------------------------------- the block -----


def _qlinear(ck: Checkpoint, stem: str, gs: int, bits: int, device, cls=QuantizedLinear):
    for suffix in ("scales", "biases"):
        if ck.dtype_of(f"{stem}.{suffix}") != "BF16":
            raise ValueError(f"{stem}.{suffix}: {ck.dtype_of(f'{stem}.{suffix}')} scales are not supported (bf16)")
    return cls(ck.tensor(f"{stem}.weight", device), ck.tensor(f"{stem}.scales", device),
               ck.tensor(f"{stem}.biases", device), gs, bits)


def load_qwen35_moe_block(model_dir: str | Checkpoint, layer: int, device="cuda") -> Qwen35MoeBlock:
    """Qwen35MoeBlock of decoder layer `layer` (moe.rs:52-78 parameters)."""
    ck = model_dir if isinstance(model_dir, Checkpoint) else Checkpoint(model_dir)
    cfg = moe_config(ck.config, layer)
    q = quantization_config(ck.config)
    p = layer_prefix(layer)
    # router: bf16, or quantised (8-bit gs64 in converted checkpoints) and expanded once
    if f"{p}.gate.scales" in ck:
        rgs, rbits = q.for_path(f"{p}.gate")
        rq = _qlinear(ck, f"{p}.gate", rgs, rbits, device)
        router = ops.dequantize(rq.weight, rq.scales, rq.biases, rgs, rbits, dtype=torch.bfloat16)
    else:
        router = ck.tensor(f"{p}.gate.weight", device)
        if router.dtype != torch.bfloat16:
            raise ValueError(f"{p}.gate.weight: router must be bf16 or quantised, got {router.dtype}")
    E, D = cfg.num_experts, cfg.hidden_size
    if tuple(router.shape) != (E, D):
        raise ValueError(f"{p}.gate: shape {tuple(router.shape)}, expected {(E, D)}")
    sw = SplitSwitchFfn(*(
        _qlinear(ck, f"{p}.switch_mlp.{n}", cfg.group_size, cfg.bits, device, QuantizedSwitchLinear)
        for n in ("gate_proj", "up_proj", "down_proj")))
    I = cfg.moe_intermediate_size
    for name, m, rows, kin in (("gate_proj", sw.gate_proj, I, D), ("up_proj", sw.up_proj, I, D),
                               ("down_proj", sw.down_proj, D, I)):
        want = (E, rows, kin * cfg.bits // 32)
        if tuple(m.weight.shape) != want:
            raise ValueError(f"{p}.switch_mlp.{name}.weight: shape {tuple(m.weight.shape)}, expected {want}")
    shared = shared_gate = None
    if cfg.shared_expert_intermediate_size:
        sb = cfg.shared_bits
        shared = SwigluMlp(*(_qlinear(ck, f"{p}.shared_expert.{n}", 64, sb, device)
                             for n in ("gate_proj", "up_proj", "down_proj")))
        shared_gate = _qlinear(ck, f"{p}.shared_expert_gate", 64, cfg.shared_gate_bits or sb, device)
    return Qwen35MoeBlock(cfg, router, sw, shared, shared_gate)


# ------------------------------------------------------------ Gemma 4 ----
# Gemma 4 checkpoints (gemma4/text/weights.rs:1-16, 60-180 of the reference's
# loader): keys under `model.language_model.layers.N` (a VLM envelope; also
# accepted: `model.layers.N`, `language_model.model.layers.N`), the router at
# `router.{proj.weight, scale, per_expert_scale}`, the experts' input norm at
# `pre_feedforward_layernorm_2.weight`, and the experts either as one
# `experts.gate_up_proj` [E, 2I, D] (dense, or quantised with
# .weight/.scales/.biases) or, as pre-quantised mlx-community checkpoints ship
# them, as `experts.{gate,up}_proj.{weight,scales,biases}`, which the
# reference concatenates along the row axis into `switch_glu.gate_up_proj`
# (merge_gate_up, weights.rs:155-180); `experts.down_proj` likewise.

_GEMMA4_PREFIXES = ("model.language_model.layers.{}", "model.layers.{}", "language_model.model.layers.{}")


def gemma4_layer_prefix(ck: "Checkpoint", layer: int) -> str:
    for f in _GEMMA4_PREFIXES:
        p = f.format(layer)
        if f"{p}.router.proj.weight" in ck:
            return p
    raise KeyError(f"layer {layer}: no Gemma 4 router (router.proj.weight) under {[f.format(layer) for f in _GEMMA4_PREFIXES]}")


def gemma4_moe_config(config: dict, bits: int, group_size: int = 64) -> MoeConfig:
    """MoeConfig (model_kind 1) of the MoE branch from config.json's text
    fields (gemma4/text/config.rs: hidden_size, num_experts, top_k_experts,
    moe_intermediate_size, rms_norm_eps)."""
    tc = text_config(config)
    if not tc.get("num_experts") or not tc.get("top_k_experts") or not tc.get("moe_intermediate_size"):
        raise ValueError("config.json describes no Gemma 4 MoE block (num_experts / top_k_experts / moe_intermediate_size)")
    if group_size != 64:
        raise ValueError(f"group size {group_size} is not supported by the block (64)")
    return MoeConfig(hidden_size=int(tc["hidden_size"]), num_experts=int(tc["num_experts"]),
                     num_experts_per_tok=int(tc["top_k_experts"]), moe_intermediate_size=int(tc["moe_intermediate_size"]),
                     group_size=group_size, bits=bits, model_kind=1, rms_norm_eps=float(tc.get("rms_norm_eps", 1e-6)))


def _bf16_vector(ck: "Checkpoint", key: str, n: int, device) -> torch.Tensor:
    t = ck.tensor(key, device)
    if tuple(t.shape) != (n,):
        raise ValueError(f"{key}: shape {tuple(t.shape)}, expected {(n,)}")
    return t.to(torch.bfloat16)


def load_gemma4_moe_branch(model_dir: str | Checkpoint, layer: int, device="cuda", bits: int = 4) -> Gemma4MoeBranch:
    """Gemma4MoeBranch of decoder layer `layer`. Quantised experts keep the
    checkpoint's group size and bits (from config.json's quantisation block);
    dense experts are quantised at load with the library's affine quantiser
    (`bits`, group 64). A quantised router projection is expanded once to
    bf16(scale * q + bias)."""
    ck = model_dir if isinstance(model_dir, Checkpoint) else Checkpoint(model_dir)
    p = gemma4_layer_prefix(ck, layer)
    q = quantization_config(ck.config)
    ex = f"{p}.experts"
    packed_q = f"{ex}.gate_up_proj.scales" in ck
    split_q = f"{ex}.gate_proj.scales" in ck
    if packed_q or split_q:
        if q is None:
            raise ValueError("quantised experts but config.json has no quantization block")
        gs, bits = q.for_path(f"{ex}.gate_up_proj" if packed_q else f"{ex}.gate_proj")
    else:
        gs = 64
    cfg = gemma4_moe_config(ck.config, bits, gs)
    E, D, I = cfg.num_experts, cfg.hidden_size, cfg.moe_intermediate_size
    # router projection
    if f"{p}.router.proj.scales" in ck:
        rgs, rbits = q.for_path(f"{p}.router.proj") if q is not None else (64, 8)
        rq = _qlinear(ck, f"{p}.router.proj", rgs, rbits, device)
        proj = ops.dequantize(rq.weight, rq.scales, rq.biases, rgs, rbits, dtype=torch.bfloat16)
    else:
        proj = ck.tensor(f"{p}.router.proj.weight", device).to(torch.bfloat16)
    if tuple(proj.shape) != (E, D):
        raise ValueError(f"{p}.router.proj: shape {tuple(proj.shape)}, expected {(E, D)}")
    # Router.scale * hidden^-0.5 in the scale's dtype (text.rs:628-639: the
    # scalar is staged into that dtype first), then bf16 for the kernel.
    scale = ck.tensor(f"{p}.router.scale", device)
    if tuple(scale.shape) != (D,):
        raise ValueError(f"{p}.router.scale: shape {tuple(scale.shape)}, expected {(D,)}")
    root = torch.tensor(D ** -0.5, dtype=torch.float32).to(scale.dtype).to(device)
    router_norm = (scale * root).to(torch.bfloat16)
    expert_scale = _bf16_vector(ck, f"{p}.router.per_expert_scale", E, device)
    experts_norm = _bf16_vector(ck, f"{p}.pre_feedforward_layernorm_2.weight", D, device)
    # experts
    if packed_q:
        gu = _qlinear(ck, f"{ex}.gate_up_proj", gs, bits, device, QuantizedSwitchLinear)
    elif split_q:
        g = _qlinear(ck, f"{ex}.gate_proj", gs, bits, device, QuantizedSwitchLinear)
        u = _qlinear(ck, f"{ex}.up_proj", gs, bits, device, QuantizedSwitchLinear)
        gu = QuantizedSwitchLinear(torch.cat([g.weight, u.weight], 1).contiguous(),
                                   torch.cat([g.scales, u.scales], 1).contiguous(),
                                   torch.cat([g.biases, u.biases], 1).contiguous(), gs, bits)
    else:
        w = ck.tensor(f"{ex}.gate_up_proj", device).to(torch.bfloat16)
        if tuple(w.shape) != (E, 2 * I, D):
            raise ValueError(f"{ex}.gate_up_proj: shape {tuple(w.shape)}, expected {(E, 2 * I, D)}")
        gu = QuantizedSwitchLinear.from_switch_linear(w, gs, bits)
    if f"{ex}.down_proj.scales" in ck:
        dn = _qlinear(ck, f"{ex}.down_proj", gs, bits, device, QuantizedSwitchLinear)
    else:
        w = ck.tensor(f"{ex}.down_proj", device).to(torch.bfloat16)
        if tuple(w.shape) != (E, D, I):
            raise ValueError(f"{ex}.down_proj: shape {tuple(w.shape)}, expected {(E, D, I)}")
        dn = QuantizedSwitchLinear.from_switch_linear(w, gs, bits)
    for name, m, rows, kin in (("gate_up_proj", gu, 2 * I, D), ("down_proj", dn, D, I)):
        want = (E, rows, kin * bits // 32)
        if tuple(m.weight.shape) != want:
            raise ValueError(f"{ex}.{name}.weight: shape {tuple(m.weight.shape)}, expected {want}")
    return Gemma4MoeBranch(cfg, proj, router_norm, expert_scale, experts_norm, PackedSwitchFfn(gu, dn))


__all__ = ["QuantizationConfig", "Checkpoint", "moe_config", "load_qwen35_moe_block", "write_safetensors",
           "read_header", "layer_prefix", "text_config", "quantization_config", "gemma4_moe_config",
           "gemma4_layer_prefix", "load_gemma4_moe_branch"]
