"""Checkpoint ingest on the CPU: config.json parsing (the quantisation block's
per-path overrides, as crates/mlxr-lm/src/quantization.rs tests them) and
the safetensors reader against files written by the module's writer."""
import json
import os

import numpy as np
import pytest

from mlxr_moe import checkpoint as ck


def test_uniform_quantization_config():
    q = ck.QuantizationConfig.from_dict({"group_size": 64, "bits": 8, "mode": "affine"})
    assert (q.group_size, q.bits, q.mode) == (64, 8, "affine")
    assert q.overrides == {}
    assert q.for_path("anything") == (64, 8)


def test_per_tensor_overrides_and_fallback():
    p0 = "language_model.model.layers.0.mlp"
    q = ck.QuantizationConfig.from_dict({
        "group_size": 64, "bits": 4, "mode": "affine",
        f"{p0}.gate": {"group_size": 64, "bits": 8},
        f"{p0}.shared_expert_gate": {"group_size": 64, "bits": 8},
    })
    assert q.bits == 4 and len(q.overrides) == 2
    assert q.for_path(f"{p0}.gate") == (64, 8)
    assert q.for_path(f"{p0}.shared_expert_gate") == (64, 8)
    assert q.for_path("language_model.model.layers.0.self_attn.q_proj") == (64, 4)


def test_default_mode_and_bad_mode():
    assert ck.QuantizationConfig.from_dict({"group_size": 32, "bits": 4}).mode == "affine"
    with pytest.raises(ValueError):
        ck.QuantizationConfig.from_dict({"group_size": 64, "bits": 4, "mode": "mxfp4"})


def _a3b_like_config(layers=2):
    """A config.json with the schema of the Qwen3.6 MoE release (text_config
    nested under a VLM envelope, router and shared-expert gate pinned at 8 bits)."""
    q = {"group_size": 64, "bits": 4, "mode": "affine"}
    for i in range(layers):
        p = f"language_model.model.layers.{i}.mlp"
        q[f"{p}.gate"] = {"group_size": 64, "bits": 8}
        q[f"{p}.shared_expert_gate"] = {"group_size": 64, "bits": 8}
    return {
        "model_type": "qwen3_5_moe",
        "text_config": {"hidden_size": 2048, "num_experts": 256, "num_experts_per_tok": 8,
                        "moe_intermediate_size": 512, "shared_expert_intermediate_size": 512,
                        "num_hidden_layers": layers},
        "quantization": q, "quantization_config": q,
    }


def test_moe_config_from_a3b_like_config():
    cfg = ck.moe_config(_a3b_like_config(), layer=1)
    assert (cfg.hidden_size, cfg.num_experts, cfg.num_experts_per_tok) == (2048, 256, 8)
    assert (cfg.moe_intermediate_size, cfg.shared_expert_intermediate_size) == (512, 512)
    assert (cfg.bits, cfg.shared_bits, cfg.shared_gate_bits, cfg.group_size) == (4, 4, 8, 64)
    c = cfg.to_c()
    assert (c.bits, c.shared_bits, c.shared_gate_bits) == (4, 4, 8)


def test_moe_config_rejects_other_group_sizes():
    c = _a3b_like_config()
    c["quantization"] = {"group_size": 32, "bits": 4}
    with pytest.raises(ValueError):
        ck.moe_config(c, 0)
    with pytest.raises(ValueError):
        ck.moe_config({"text_config": c["text_config"]}, 0)  # no quantisation block


def test_safetensors_round_trip_sharded(tmp_path):
    rng = np.random.default_rng(0)
    a = rng.integers(0, 2**32, size=(4, 8, 16), dtype=np.uint32)
    b = rng.integers(0, 2**16, size=(4, 8, 2), dtype=np.uint16)  # bf16 bit patterns
    c = rng.standard_normal((3, 5)).astype(np.float32)
    ck.write_safetensors(str(tmp_path / "model-00001-of-00002.safetensors"), {"x.weight": a, "x.scales": b})
    ck.write_safetensors(str(tmp_path / "model-00002-of-00002.safetensors"), {"y": c})
    with open(tmp_path / "model.safetensors.index.json", "w") as f:
        json.dump({"metadata": {"total_size": a.nbytes + b.nbytes + c.nbytes},
                   "weight_map": {"x.weight": "model-00001-of-00002.safetensors",
                                  "x.scales": "model-00001-of-00002.safetensors",
                                  "y": "model-00002-of-00002.safetensors"}}, f)
    with open(tmp_path / "config.json", "w") as f:
        json.dump(_a3b_like_config(), f)
    m = ck.Checkpoint(str(tmp_path))
    assert "x.weight" in m and "nope" not in m
    np.testing.assert_array_equal(m.numpy("x.weight"), a)
    np.testing.assert_array_equal(m.numpy("x.scales"), b)
    assert m.dtype_of("x.scales") == "BF16"
    np.testing.assert_array_equal(m.numpy("y"), c)
    header, base = ck.read_header(str(tmp_path / "model-00002-of-00002.safetensors"))
    assert base % 8 == 0 and header["y"]["shape"] == [3, 5] and header["y"]["dtype"] == "F32"
    with pytest.raises(KeyError):
        m.numpy("nope")


def test_single_file_checkpoint(tmp_path):
    v = np.arange(12, dtype=np.uint32).reshape(3, 4)
    ck.write_safetensors(str(tmp_path / "model.safetensors"), {"w": v})
    with open(tmp_path / "config.json", "w") as f:
        json.dump({}, f)
    m = ck.Checkpoint(str(tmp_path))
    np.testing.assert_array_equal(m.numpy("w"), v)
    os.remove(tmp_path / "model.safetensors")
    with pytest.raises(FileNotFoundError):
        ck.Checkpoint(str(tmp_path))


def _gemma4_config():
    return {"model_type": "gemma4", "text_config": {"hidden_size": 2048, "num_experts": 128, "top_k_experts": 8,
                                                    "moe_intermediate_size": 768, "rms_norm_eps": 1e-6,
                                                    "enable_moe_block": True},
            "quantization": {"group_size": 64, "bits": 4, "mode": "affine"}}


def test_gemma4_moe_config():
    cfg = ck.gemma4_moe_config(_gemma4_config(), bits=4)
    assert (cfg.hidden_size, cfg.num_experts, cfg.num_experts_per_tok, cfg.moe_intermediate_size) == (2048, 128, 8, 768)
    assert cfg.model_kind == 1 and cfg.shared_expert_intermediate_size == 0 and abs(cfg.rms_norm_eps - 1e-6) < 1e-12
    c = cfg.to_c()
    assert c.model_kind == 1 and abs(c.rms_norm_eps - 1e-6) < 1e-9
    with pytest.raises(ValueError):
        ck.gemma4_moe_config({"text_config": {"hidden_size": 2048}}, bits=4)  # a dense-MLP model
    with pytest.raises(ValueError):
        ck.gemma4_moe_config(_gemma4_config(), bits=4, group_size=32)


@pytest.mark.parametrize("prefix", ["model.language_model.layers.5", "model.layers.5", "language_model.model.layers.5"])
def test_gemma4_layer_prefix(tmp_path, prefix):
    ck.write_safetensors(str(tmp_path / "model.safetensors"),
                         {f"{prefix}.router.proj.weight": np.zeros((4, 8), np.uint16)}, {f"{prefix}.router.proj.weight": "BF16"})
    with open(tmp_path / "config.json", "w") as f:
        json.dump(_gemma4_config(), f)
    m = ck.Checkpoint(str(tmp_path))
    assert ck.gemma4_layer_prefix(m, 5) == prefix
    with pytest.raises(KeyError):
        ck.gemma4_layer_prefix(m, 6)
