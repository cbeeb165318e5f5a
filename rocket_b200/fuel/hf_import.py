"""Import a Hugging Face checkpoint (GLM-4.x MoE, Qwen3-Next, Qwen3 MoE) as a fuel.

    python -m rocket_b200 import-hf --src hf_dir --out fuel_dir [--id my-fuel]
    python -m rocket_b200 quantize-fuel --src fuel_dir --out nvfp4_dir --fuel fuel_dir/fuel.yaml

Tensor names map onto the fuel names (models/weights.py) and three weights change
row order, because the fuel keeps contiguous blocks where the HF modules interleave
per head group:

* gated attention ``q_proj`` (Qwen3-Next): HF rows are [q_h | gate_h] per head
  (the module views the output as (heads, 2*head_dim) and chunks it); the fuel
  holds [all q | all gate];
* DeltaNet ``in_proj_qkvz``: HF rows are grouped per key head, [q_h, k_h, v_h, z_h]
  with r = Hv/Hk value heads in v_h and z_h; the fuel holds [Q | K | V | Z];
* DeltaNet ``in_proj_ba``: HF rows per key head [b (r) | a (r)]; the fuel [B | A].

Row permutations apply to bf16 weights and to both NVFP4 row tensors (``.weight``,
``.weight_scale``) alike, so an NVFP4 (ModelOpt-layout) checkpoint imports as is.
The conv1d weight [C, 1, K] loses its middle axis; rotary buffers and the MTP
layer's copies of the embedding / lm_head are dropped.  Conversion streams one
input shard at a time.  The layouts above are those of the public transformers
modules for these model types; the engine refuses a checkpoint whose config.json
disagrees with the fuel (config/hf.py).
"""
from __future__ import annotations

import json
import os
import re

import torch

from ..config.hf import SUPPORTED, fuel_yaml_from_hf, model_config_from_hf

_LAYER = re.compile(r"^model\.layers\.(\d+)\.(.+)$")
_W = r"(weight|weight_scale|weight_scale_2)"  # a bf16 weight or an NVFP4 triplet
_COMMON = [
    (r"^input_layernorm\.weight$", r"attn_norm.weight"),
    (r"^post_attention_layernorm\.weight$", r"mlp_norm.weight"),
    (r"^self_attn\.(q_norm|k_norm)\.weight$", r"attn.\1.weight"),
    (r"^self_attn\.(q_proj|k_proj|v_proj|o_proj)\." + _W + "$", r"attn.\1.\2"),
    (r"^self_attn\.(q_proj|k_proj|v_proj)\.bias$", r"attn.\1.bias"),
    (r"^mlp\.experts\.(\d+)\.(gate_proj|up_proj|down_proj)\." + _W + "$", r"moe.experts.\1.\2.\3"),
    (r"^mlp\.gate\.weight$", r"moe.router.weight"),
    (r"^mlp\.gate\.e_score_correction_bias$", r"moe.router.bias"),
    (r"^mlp\.shared_experts?\.(gate_proj|up_proj|down_proj)\." + _W + "$", r"moe.shared.\1.\2"),
    (r"^mlp\.shared_expert_gate\.weight$", r"moe.shared_gate.weight"),
    (r"^mlp\.(gate_proj|up_proj|down_proj)\." + _W + "$", r"mlp.\1.\2"),
    (r"^linear_attn\.(in_proj_qkvz|in_proj_ba|out_proj)\." + _W + "$", r"dn.\1.\2"),
    (r"^linear_attn\.norm\.weight$", r"dn.norm.weight"),
    (r"^linear_attn\.conv1d\.weight$", r"dn.conv1d.weight"),
    (r"^linear_attn\.(A_log|dt_bias)$", r"dn.\1"),
]
_COMMON = [(re.compile(a), b) for a, b in _COMMON]


def _layer_suffix(rest: str) -> str | None:
    for pat, rep in _COMMON:
        if pat.match(rest):
            return pat.sub(rep, rest)
    return None


def fuel_name(name: str, cfg: dict) -> str | None:
    """Fuel name of HF tensor `name` (None: not carried over).  Raises on a tensor the
    fuel has no place for (so nothing is silently dropped)."""
    if name.endswith(("rotary_emb.inv_freq", ".input_scale")):
        return None  # rotary buffers; activation calibration scales (NVFP4 activations are dynamic here)
    if name == "model.embed_tokens.weight":
        return "embed.weight"
    if name == "model.norm.weight":
        return "final_norm.weight"
    if name.startswith("lm_head."):
        return name
    L = cfg["num_hidden_layers"]
    m = _LAYER.match(name)
    if m:
        i, rest = int(m.group(1)), m.group(2)
        if i < L:
            s = _layer_suffix(rest)
            if s is None:
                raise ValueError(f"{name}: no fuel tensor for it")
            return f"layers.{i}.{s}"
        j = i - L  # GLM-style MTP layers follow the decoder layers
        if rest in ("embed_tokens.weight", "shared_head.head.weight") or rest.startswith("shared_head.head."):
            return None  # shared with the main model
        for k, v in (("eh_proj.", "eh_proj."), ("enorm.", "enorm."), ("hnorm.", "hnorm."),
                     ("shared_head.norm.", "norm.")):
            if rest.startswith(k):
                return f"mtp.{j}.{v}{rest[len(k):]}"
        s = _layer_suffix(rest)
        if s is None:
            raise ValueError(f"{name}: no fuel tensor for it")
        return f"mtp.{j}.layer.{s}"
    if name.startswith("mtp."):  # Qwen3-Next MTP module
        rest = name[4:]
        for k, v in (("fc.", "eh_proj."), ("pre_fc_norm_embedding.", "enorm."), ("pre_fc_norm_hidden.", "hnorm."),
                     ("norm.", "norm.")):
            if rest.startswith(k):
                return f"mtp.0.{v}{rest[len(k):]}"
        mm = re.match(r"^layers\.(\d+)\.(.+)$", rest)
        if mm:
            s = _layer_suffix(mm.group(2))
            if s is not None:
                return f"mtp.{mm.group(1)}.layer.{s}"
    raise ValueError(f"{name}: no fuel tensor for it")


def _perm_gated_q(heads: int, hd: int) -> torch.Tensor:
    """HF row order [q_h | g_h] per head -> fuel [all q | all gate]: fuel row i takes HF row perm[i]."""
    h = torch.arange(heads)[:, None] * 2 * hd
    q = (h + torch.arange(hd)[None, :]).reshape(-1)
    g = (h + hd + torch.arange(hd)[None, :]).reshape(-1)
    return torch.cat([q, g])


def _perm_qkvz(hk: int, hv: int, dk: int, dv: int) -> torch.Tensor:
    r = hv // hk
    grp = 2 * dk + 2 * r * dv
    base = torch.arange(hk)[:, None] * grp
    q = (base + torch.arange(dk)).reshape(-1)
    k = (base + dk + torch.arange(dk)).reshape(-1)
    v = (base + 2 * dk + torch.arange(r * dv)).reshape(-1)
    z = (base + 2 * dk + r * dv + torch.arange(r * dv)).reshape(-1)
    return torch.cat([q, k, v, z])


def _perm_ba(hk: int, hv: int) -> torch.Tensor:
    r = hv // hk
    base = torch.arange(hk)[:, None] * 2 * r
    b = (base + torch.arange(r)).reshape(-1)
    a = (base + r + torch.arange(r)).reshape(-1)
    return torch.cat([b, a])


def row_permutation(fuel: str, cfg: dict) -> torch.Tensor | None:
    """Rows to gather from the HF tensor for fuel tensor `fuel` (None: unchanged)."""
    base = fuel.rsplit(".", 1)[0] if fuel.endswith((".weight", ".weight_scale", ".bias")) else None
    if base is None:
        return None
    mt = cfg["model_type"]
    if mt == "qwen3_next" and base.endswith("attn.q_proj"):
        hd = cfg.get("head_dim") or cfg["hidden_size"] // cfg["num_attention_heads"]
        return _perm_gated_q(cfg["num_attention_heads"], hd)
    if base.endswith("dn.in_proj_qkvz"):
        return _perm_qkvz(cfg["linear_num_key_heads"], cfg["linear_num_value_heads"], cfg["linear_key_head_dim"],
                          cfg["linear_value_head_dim"])
    if base.endswith("dn.in_proj_ba"):
        return _perm_ba(cfg["linear_num_key_heads"], cfg["linear_num_value_heads"])
    return None


def convert(tensors: dict, cfg: dict) -> dict:
    """HF-named tensors -> fuel-named tensors (renamed, reordered)."""
    if cfg.get("model_type") not in SUPPORTED:
        raise ValueError(f"model_type {cfg.get('model_type')!r} is not one of {SUPPORTED}")
    out = {}
    for name, t in tensors.items():
        f = fuel_name(name, cfg)
        if f is None:
            continue
        p = row_permutation(f, cfg)
        if p is not None:
            if t.shape[0] != p.numel():
                raise ValueError(f"{name}: {t.shape[0]} rows, the layout needs {p.numel()}")
            t = t.index_select(0, p).contiguous()
        if f.endswith("dn.conv1d.weight") and t.dim() == 3:
            t = t[:, 0, :].contiguous()
        out[f] = t
    return out


def import_hf(src: str, out_dir: str, fuel_id: str | None = None) -> dict:
    """Convert an HF checkpoint directory shard by shard into a fuel directory
    (fuel-named safetensors + index + fuel.yaml).  Returns a small report."""
    from .safetensors_io import INDEX, load_file, save_file
    with open(os.path.join(src, "config.json")) as f:
        cfg = json.load(f)
    model_config_from_hf(cfg)  # refuses unsupported configs before any work
    os.makedirs(out_dir, exist_ok=True)
    idx_path = os.path.join(src, INDEX)
    if os.path.exists(idx_path):
        with open(idx_path) as f:
            shards = sorted(set(json.load(f)["weight_map"].values()))
    else:
        shards = sorted(x for x in os.listdir(src) if x.endswith(".safetensors"))
    weight_map, n = {}, 0
    for k, sh in enumerate(shards):
        conv = convert(load_file(os.path.join(src, sh)), cfg)
        name = f"model-{k + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(conv, os.path.join(out_dir, name))
        weight_map.update({t: name for t in conv})
        n += len(conv)
    with open(os.path.join(out_dir, INDEX), "w") as f:
        json.dump({"metadata": {"source": os.path.abspath(src)}, "weight_map": weight_map}, f, indent=1)
    fid = fuel_id or cfg.get("model_type")
    with open(os.path.join(out_dir, "fuel.yaml"), "w") as f:
        f.write(fuel_yaml_from_hf(cfg, fid))
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    return {"tensors": n, "shards": len(shards), "fuel": os.path.join(out_dir, "fuel.yaml")}
