"""HF checkpoint import: fuel tensors written out in the HF module layouts (names,
per-head-group row interleaves, conv1d [C, 1, K], MTP placement) import back to the
same fuel tensors, for a Qwen3-Next-style and a GLM-style model; the directory import
streams shards and writes a fuel.yaml whose config matches."""
import json

import pytest
import torch

from rocket_b200.config import load_fuel
from rocket_b200.config.hf import hf_mismatches
from rocket_b200.fuel.hf_import import convert, fuel_name, import_hf
from rocket_b200.models import init_fuel_tensors


def _hf_cfg(m, mt):
    c = {"model_type": mt, "hidden_size": m.d_model, "num_hidden_layers": m.num_layers,
         "num_attention_heads": m.num_q_heads, "num_key_value_heads": m.num_kv_heads, "head_dim": m.head_dim,
         "partial_rotary_factor": m.rotary_fraction, "rope_theta": m.rope_theta, "rms_norm_eps": m.norm_eps,
         "vocab_size": m.vocab_size, "norm_topk_prob": m.norm_topk_prob, "moe_intermediate_size": m.moe_intermediate,
         "num_experts_per_tok": m.top_k, "tie_word_embeddings": False, "num_nextn_predict_layers": m.mtp_layers}
    if mt == "qwen3_next":
        dn = m.deltanet
        c.update(num_experts=m.num_experts, shared_expert_intermediate_size=m.shared_intermediate,
                 full_attention_interval=len(m.layer_pattern), linear_num_key_heads=dn.num_qk_heads,
                 linear_num_value_heads=dn.num_v_heads, linear_key_head_dim=dn.head_dim,
                 linear_value_head_dim=dn.head_dim, linear_conv_kernel_dim=dn.conv_kernel, decoder_sparse_step=1,
                 mlp_only_layers=[])
    else:
        c.update(n_routed_experts=m.num_experts, n_shared_experts=m.num_shared_experts,
                 first_k_dense_replace=m.num_dense_layers, intermediate_size=m.dense_intermediate,
                 routed_scaling_factor=m.routed_scaling, use_qk_norm=m.qk_norm)
    return c


def _to_hf(t, m, cfg):
    """The inverse of the import, written from the HF module layouts."""
    L = m.num_layers
    out = {}
    for name, x in t.items():
        if name.startswith("master."):
            continue
        if name == "embed.weight":
            hn = "model.embed_tokens.weight"
        elif name == "final_norm.weight":
            hn = "model.norm.weight"
        elif name.startswith("lm_head"):
            hn = name
        else:
            if name.startswith("mtp."):
                _, j, rest = name.split(".", 2)
                if cfg["model_type"] == "qwen3_next":
                    top = {"eh_proj": "mtp.fc", "enorm": "mtp.pre_fc_norm_embedding",
                           "hnorm": "mtp.pre_fc_norm_hidden", "norm": "mtp.norm"}
                    head, _, tail = rest.partition(".")
                    if head in top:
                        out[f"{top[head]}.{tail}"] = x
                        continue
                    prefix, rest = f"mtp.layers.{j}.", rest[len("layer."):]
                else:
                    head, _, tail = rest.partition(".")
                    top = {"eh_proj": "eh_proj", "enorm": "enorm", "hnorm": "hnorm", "norm": "shared_head.norm"}
                    if head in top:
                        out[f"model.layers.{L + int(j)}.{top[head]}.{tail}"] = x
                        continue
                    prefix, rest = f"model.layers.{L + int(j)}.", rest[len("layer."):]
            else:
                _, i, rest = name.split(".", 2)
                prefix = f"model.layers.{i}."
            rest = (rest.replace("attn_norm.", "input_layernorm.").replace("mlp_norm.", "post_attention_layernorm.")
                    .replace("attn.", "self_attn.").replace("moe.router.weight", "mlp.gate.weight")
                    .replace("moe.router.bias", "mlp.gate.e_score_correction_bias")
                    .replace("moe.experts.", "mlp.experts.").replace("moe.shared_gate.", "mlp.shared_expert_gate.")
                    .replace("moe.shared.", "mlp.shared_expert." if cfg["model_type"] == "qwen3_next"
                             else "mlp.shared_experts.")
                    .replace("dn.", "linear_attn."))
            hn = prefix + rest
            if rest.startswith("linear_attn.conv1d"):
                x = x[:, None, :]
            base = rest.rsplit(".", 1)[0]
            if rest.endswith((".weight", ".weight_scale")) and base in ("self_attn.q_proj", "linear_attn.in_proj_qkvz",
                                                                        "linear_attn.in_proj_ba"):
                x = _interleave(x, base, m, cfg)
        out[hn] = x
    if cfg["model_type"] == "glm4_moe" and m.mtp_layers:
        out[f"model.layers.{L}.embed_tokens.weight"] = t["embed.weight"]
    out["model.layers.0.self_attn.rotary_emb.inv_freq"] = torch.ones(4)
    return out


def _interleave(x, base, m, cfg):
    if base == "self_attn.q_proj":
        if not m.attn_output_gate:
            return x
        H, D = m.num_q_heads, m.head_dim
        q, g = x[:H * D].reshape(H, D, *x.shape[1:]), x[H * D:].reshape(H, D, *x.shape[1:])
        return torch.stack([q, g], 1).reshape(x.shape)
    dn = m.deltanet
    hk, hv, dk = dn.num_qk_heads, dn.num_v_heads, dn.head_dim
    r = hv // hk
    if base.endswith("in_proj_ba"):
        b, a = x[:hv].reshape(hk, r, *x.shape[1:]), x[hv:].reshape(hk, r, *x.shape[1:])
        return torch.cat([b, a], 1).reshape(x.shape)
    q = x[:hk * dk].reshape(hk, dk, *x.shape[1:])
    k = x[hk * dk:2 * hk * dk].reshape(hk, dk, *x.shape[1:])
    v = x[2 * hk * dk:2 * hk * dk + hv * dk].reshape(hk, r * dk, *x.shape[1:])
    z = x[2 * hk * dk + hv * dk:].reshape(hk, r * dk, *x.shape[1:])
    return torch.cat([q, k, v, z], 1).reshape(x.shape)


@pytest.mark.parametrize("fuel,mt", [("tiny-hybrid", "qwen3_next"), ("glm-moe-small", "glm4_moe")])
def test_hf_layout_imports_back_to_the_fuel(fuel, mt):
    m = load_fuel(fuel).model
    t = init_fuel_tensors(m, 0)
    cfg = _hf_cfg(m, mt)
    assert hf_mismatches(m, cfg) == []
    back = convert(_to_hf(t, m, cfg), cfg)
    want = {k: v for k, v in t.items() if not k.startswith("master.")}
    assert set(back) == set(want)
    for k in want:
        assert back[k].dtype == want[k].dtype and torch.equal(back[k], want[k]), k


def test_unknown_tensors_are_refused():
    m = load_fuel("glm-moe-small").model
    cfg = _hf_cfg(m, "glm4_moe")
    with pytest.raises(ValueError, match="no fuel tensor"):
        fuel_name("model.layers.0.self_attn.q_proj.bias_extra", cfg)
    with pytest.raises(ValueError, match="model_type"):
        convert({}, dict(cfg, model_type="llama"))


def test_import_directory(tmp_path):
    from rocket_b200.fuel.safetensors_io import load_dir, save_file
    m = load_fuel("tiny-hybrid").model
    t = init_fuel_tensors(m, 1)
    cfg = _hf_cfg(m, "qwen3_next")
    hf = _to_hf(t, m, cfg)
    src = tmp_path / "hf"
    src.mkdir()
    names = sorted(hf)
    save_file({k: hf[k] for k in names[:len(names) // 2]}, str(src / "a.safetensors"))
    save_file({k: hf[k] for k in names[len(names) // 2:]}, str(src / "b.safetensors"))
    (src / "config.json").write_text(json.dumps(cfg))
    rep = import_hf(str(src), str(tmp_path / "fuel"), "tiny-next")
    assert rep["shards"] == 2
    back = load_dir(str(tmp_path / "fuel"))
    want = {k: v for k, v in t.items() if not k.startswith("master.")}
    assert set(back) == set(want) and all(torch.equal(back[k], want[k]) for k in want)
    fm = load_fuel(rep["fuel"]).model
    assert fm.name == "tiny-next" and hf_mismatches(fm, cfg) == []


def test_attention_biases_import():
    from rocket_b200.config.schema import model_config
    m = model_config("glm-moe-small", attention_bias=True)
    t = init_fuel_tensors(m, 0)
    cfg = dict(_hf_cfg(m, "glm4_moe"), attention_bias=True)
    assert hf_mismatches(m, cfg) == []
    assert hf_mismatches(load_fuel("glm-moe-small").model, cfg) == ["attention_bias: fuel False != checkpoint True"]
    hf = _to_hf(t, m, cfg)
    assert "model.layers.0.self_attn.q_proj.bias" in hf
    back = convert(hf, cfg)
    want = {k: v for k, v in t.items() if not k.startswith("master.")}
    assert set(back) == set(want) and all(torch.equal(back[k], want[k]) for k in want)


def test_cli_fuel_from_hf_and_import(tmp_path):
    """A bf16 HF checkpoint through the command lines: fuel-from-hf, import-hf, then
    quantize-fuel (NVFP4 experts per the generated fuel.yaml) and verify-fuel."""
    import subprocess
    import sys

    from rocket_b200.fuel.safetensors_io import load_dir, save_file
    m = load_fuel("tiny-hybrid").model
    t = init_fuel_tensors(m, 3)
    bf = {}  # the unquantized (bf16) checkpoint behind the fuel tensors
    for k, v in t.items():
        if k.startswith("master.") or k.endswith((".weight_scale", ".weight_scale_2")):
            continue
        base = k[:-len(".weight")] if k.endswith(".weight") else None
        bf[k] = t["master." + base].bfloat16() if base and "master." + base in t else v
    cfg = _hf_cfg(m, "qwen3_next")
    src = tmp_path / "hf"
    src.mkdir()
    save_file(_to_hf(bf, m, cfg), str(src / "model.safetensors"))
    (src / "config.json").write_text(json.dumps(cfg))
    run = lambda *a: subprocess.run([sys.executable, "-m", "rocket_b200", *a], capture_output=True, text=True,
                                    timeout=600)
    out = run("fuel-from-hf", "--config", str(src / "config.json"), "--id", "cli-next")
    assert out.returncode == 0 and "id: cli-next" in out.stdout, out.stderr[-800:]
    out = run("import-hf", "--src", str(src), "--out", str(tmp_path / "fuel"), "--id", "cli-next")
    assert out.returncode == 0, out.stderr[-800:]
    rep = json.loads(out.stdout.strip().splitlines()[-1])
    back = load_dir(str(tmp_path / "fuel"))
    assert rep["tensors"] == len(back) == len(bf)
    assert all(torch.equal(back[k], bf[k]) for k in bf)
    out = run("quantize-fuel", "--src", str(tmp_path / "fuel"), "--out", str(tmp_path / "nv"), "--fuel", rep["fuel"])
    assert out.returncode == 0, out.stderr[-800:]
    nv = load_dir(str(tmp_path / "nv"))
    e0 = "layers.0.moe.experts.0.gate_proj"
    assert nv[e0 + ".weight"].dtype == torch.uint8 and e0 + ".weight_scale" in nv and e0 + ".weight_scale_2" in nv
    out = run("verify-fuel", "--dir", str(tmp_path / "nv"))
    assert out.returncode == 0, out.stdout[-800:] + out.stderr[-800:]
