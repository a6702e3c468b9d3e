"""Qwen 3.5 / 3.6 MoE blocks from an mlxr-convert checkpoint directory.

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
from .moe import MoeConfig, QuantizedLinear, QuantizedSwitchLinear, Qwen35MoeBlock, SplitSwitchFfn, SwigluMlp

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


__all__ = ["QuantizationConfig", "Checkpoint", "moe_config", "load_qwen35_moe_block", "write_safetensors",
           "read_header", "layer_prefix", "text_config", "quantization_config"]
