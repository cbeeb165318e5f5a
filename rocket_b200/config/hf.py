"""Hugging Face ``config.json`` <-> fuel model config.

``model_config_from_hf(cfg)`` derives a ModelConfig from the config.json of a GLM-4.x
MoE (``glm4_moe``), Qwen3-Next (``qwen3_next``) or Qwen3 MoE (``qwen3_moe``)
checkpoint; ``hf_mismatches(model, cfg)`` lists every architecture field on which a
fuel disagrees with a checkpoint's config.json, and the engine refuses to load a
checkpoint directory whose config.json disagrees with the fuel (fail-closed, as the
reference's model config loader does when attention.yaml and config.json disagree:
engines/glm5-moe-nvfp4-2b/src/model_config.h:1-9).

    python -m rocket_b200 fuel-from-hf --config ckpt/config.json --out fuels/mine.yaml
"""
from __future__ import annotations

import dataclasses
import json
import os

from .schema import ConfigError, DeltaNetConfig, ModelConfig

SUPPORTED = ("glm4_moe", "qwen3_next", "qwen3_moe")


def _get(cfg: dict, *keys, default=None):
    for k in keys:
        if k in cfg and cfg[k] is not None:
            return cfg[k]
    return default


def model_config_from_hf(cfg: dict, name: str | None = None) -> ModelConfig:
    """ModelConfig of a supported config.json (weight formats keep the fuel defaults:
    NVFP4 experts / dense MLPs, bf16 attention and lm_head)."""
    mt = cfg.get("model_type")
    if mt not in SUPPORTED:
        raise ConfigError(f"config.json model_type {mt!r} is not one of {SUPPORTED}")
    d = cfg["hidden_size"]
    nq = cfg["num_attention_heads"]
    base = dict(
        name=name or cfg.get("_name_or_path") or mt,
        vocab_size=cfg["vocab_size"], num_layers=cfg["num_hidden_layers"], d_model=d, num_q_heads=nq,
        num_kv_heads=_get(cfg, "num_key_value_heads", default=nq),
        head_dim=_get(cfg, "head_dim", default=d // nq),
        rope_theta=float(_get(cfg, "rope_theta", default=10000.0)),
        rotary_fraction=float(_get(cfg, "partial_rotary_factor", default=1.0)),
        norm_eps=float(_get(cfg, "rms_norm_eps", default=1e-6)),
        norm_topk_prob=bool(_get(cfg, "norm_topk_prob", default=True)),
        tie_embeddings=bool(_get(cfg, "tie_word_embeddings", default=False)),
        attention_bias=bool(_get(cfg, "attention_bias", default=False)),
        mtp_layers=int(_get(cfg, "num_nextn_predict_layers", "mtp_num_hidden_layers", default=0)),
    )
    if mt == "glm4_moe":
        base.update(
            num_dense_layers=int(_get(cfg, "first_k_dense_replace", default=0)),
            dense_intermediate=cfg["intermediate_size"], num_experts=cfg["n_routed_experts"],
            moe_intermediate=cfg["moe_intermediate_size"], top_k=cfg["num_experts_per_tok"], router="sigmoid",
            routed_scaling=float(_get(cfg, "routed_scaling_factor", default=1.0)),
            num_shared_experts=int(_get(cfg, "n_shared_experts", default=0)),
            shared_intermediate=cfg["moe_intermediate_size"] * max(1, int(_get(cfg, "n_shared_experts", default=1))),
            qk_norm=bool(_get(cfg, "use_qk_norm", default=False)), layer_pattern=["attention"])
    elif mt == "qwen3_moe":
        base.update(
            num_experts=cfg["num_experts"], moe_intermediate=cfg["moe_intermediate_size"],
            top_k=cfg["num_experts_per_tok"], router="softmax", num_shared_experts=0, shared_intermediate=0,
            qk_norm=True, layer_pattern=["attention"],
            num_dense_layers=0, dense_intermediate=_get(cfg, "intermediate_size", default=0))
        if _get(cfg, "mlp_only_layers", default=[]) or int(_get(cfg, "decoder_sparse_step", default=1)) != 1:
            raise ConfigError("qwen3_moe: mlp_only_layers / decoder_sparse_step != 1 are not supported")
    else:  # qwen3_next
        interval = int(_get(cfg, "full_attention_interval", default=4))
        types = cfg.get("layer_types")
        if types:
            pattern = ["attention" if t == "full_attention" else "deltanet" for t in types]
            period = next((p for p in range(1, len(pattern) + 1)
                           if all(pattern[i] == pattern[i % p] for i in range(len(pattern)))), len(pattern))
            pattern = pattern[:period]
        else:
            pattern = ["deltanet"] * (interval - 1) + ["attention"]
        if int(_get(cfg, "linear_key_head_dim", default=128)) != int(_get(cfg, "linear_value_head_dim", default=128)):
            raise ConfigError("qwen3_next: DeltaNet key and value head dims must be equal")
        if _get(cfg, "mlp_only_layers", default=[]) or int(_get(cfg, "decoder_sparse_step", default=1)) != 1:
            raise ConfigError("qwen3_next: mlp_only_layers / decoder_sparse_step != 1 are not supported")
        base.update(
            num_experts=cfg["num_experts"], moe_intermediate=cfg["moe_intermediate_size"],
            top_k=cfg["num_experts_per_tok"], router="softmax", num_shared_experts=1,
            shared_intermediate=_get(cfg, "shared_expert_intermediate_size", default=cfg["moe_intermediate_size"]),
            shared_expert_gate=True, layer_pattern=pattern, attn_output_gate=True, qk_norm=True,
            zero_centered_norm=True,
            deltanet=DeltaNetConfig(num_qk_heads=cfg["linear_num_key_heads"],
                                    num_v_heads=cfg["linear_num_value_heads"],
                                    head_dim=int(_get(cfg, "linear_key_head_dim", default=128)),
                                    conv_kernel=int(_get(cfg, "linear_conv_kernel_dim", default=4))))
    return ModelConfig(**base).validate()


# fields a checkpoint fixes (weight formats, init and serving knobs are the fuel's own)
_ARCH_FIELDS = ("vocab_size", "num_layers", "d_model", "num_q_heads", "num_kv_heads", "head_dim", "rope_theta",
                "rotary_fraction", "norm_eps", "num_dense_layers", "dense_intermediate", "num_experts",
                "moe_intermediate", "top_k", "router", "norm_topk_prob", "routed_scaling", "num_shared_experts",
                "shared_intermediate", "shared_expert_gate", "layer_pattern", "attn_output_gate", "qk_norm",
                "zero_centered_norm", "deltanet", "tie_embeddings", "attention_bias")


def hf_mismatches(model: ModelConfig, cfg: dict) -> list[str]:
    """Architecture fields on which `model` disagrees with config.json `cfg`
    (the MTP depth and layer count are checked as `model` <= checkpoint: a fuel may
    serve fewer MTP layers, or fewer layers of a checkpoint cut for a test)."""
    ref = model_config_from_hf(cfg)
    out = []
    for f in _ARCH_FIELDS:
        a, b = getattr(model, f), getattr(ref, f)
        if dataclasses.is_dataclass(a) or dataclasses.is_dataclass(b):
            a = dataclasses.asdict(a) if a is not None else None
            b = dataclasses.asdict(b) if b is not None else None
            if a and b:  # gate options are fuel-side choices
                a = {k: v for k, v in a.items() if k in ("num_qk_heads", "num_v_heads", "head_dim", "conv_kernel")}
                b = {k: v for k, v in b.items() if k in a}
        if f == "num_layers":
            if a > b:
                out.append(f"num_layers: fuel {a} > checkpoint {b}")
            continue
        if isinstance(a, float) or isinstance(b, float):
            if abs(float(a) - float(b)) > 1e-9 * max(1.0, abs(float(b))):
                out.append(f"{f}: fuel {a} != checkpoint {b}")
        elif a != b:
            out.append(f"{f}: fuel {a} != checkpoint {b}")
    if model.mtp_layers > ref.mtp_layers:
        out.append(f"mtp_layers: fuel {model.mtp_layers} > checkpoint {ref.mtp_layers}")
    return out


def check_checkpoint_dir(model: ModelConfig, fuel_dir: str) -> None:
    """Refuse a checkpoint directory whose config.json disagrees with the fuel (no
    config.json: nothing to check)."""
    p = os.path.join(fuel_dir, "config.json")
    if not os.path.exists(p):
        return
    with open(p) as f:
        cfg = json.load(f)
    if cfg.get("model_type") not in SUPPORTED:
        return
    bad = hf_mismatches(model, cfg)
    if bad:
        raise ConfigError(f"{p} disagrees with the fuel: " + "; ".join(bad))


def fuel_yaml_from_hf(cfg: dict, fuel_id: str) -> str:
    """A fuel YAML document for config.json `cfg`."""
    import yaml
    m = model_config_from_hf(cfg, name=fuel_id)
    d = dataclasses.asdict(m)
    for k in ("deltanet", "mla", "sparse_attention"):
        if d.get(k) is None:
            d.pop(k, None)
    doc = {"id": fuel_id, "chemistry": cfg.get("model_type"), "status": "from config.json",
           "notes": "derived by fuel-from-hf; weight formats are the fuel defaults", "model": d}
    return yaml.safe_dump(doc, sort_keys=False)
