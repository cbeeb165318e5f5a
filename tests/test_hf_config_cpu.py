"""config.json <-> fuel: derivation for the supported families, the mismatch list the
engine refuses a checkpoint on, and the generated fuel YAML round trip."""
import json

import pytest

from rocket_b200.config import load_fuel
from rocket_b200.config.hf import check_checkpoint_dir, fuel_yaml_from_hf, hf_mismatches, model_config_from_hf
from rocket_b200.config.schema import ConfigError

QWEN3_NEXT = {"model_type": "qwen3_next", "hidden_size": 2048, "num_hidden_layers": 48, "num_attention_heads": 16,
              "num_key_value_heads": 2, "head_dim": 256, "partial_rotary_factor": 0.25, "rope_theta": 10000000,
              "rms_norm_eps": 1e-6, "vocab_size": 151936, "full_attention_interval": 4, "linear_conv_kernel_dim": 4,
              "linear_key_head_dim": 128, "linear_value_head_dim": 128, "linear_num_key_heads": 16,
              "linear_num_value_heads": 32, "num_experts": 512, "num_experts_per_tok": 10,
              "moe_intermediate_size": 512, "shared_expert_intermediate_size": 512, "norm_topk_prob": True,
              "decoder_sparse_step": 1, "mlp_only_layers": [], "intermediate_size": 5120,
              "tie_word_embeddings": False, "num_nextn_predict_layers": 1}
GLM = {"model_type": "glm4_moe", "hidden_size": 5120, "num_hidden_layers": 60, "num_attention_heads": 96,
       "num_key_value_heads": 8, "head_dim": 128, "partial_rotary_factor": 1.0, "rope_theta": 1000000,
       "rms_norm_eps": 1e-5, "vocab_size": 151552, "first_k_dense_replace": 3, "intermediate_size": 12288,
       "moe_intermediate_size": 1536, "n_routed_experts": 160, "n_shared_experts": 1, "num_experts_per_tok": 8,
       "norm_topk_prob": True, "routed_scaling_factor": 1.0, "use_qk_norm": False, "num_nextn_predict_layers": 1,
       "tie_word_embeddings": False}


@pytest.mark.parametrize("fuel,cfg", [("qwen3-next-hybrid", QWEN3_NEXT), ("glm-moe-355b", GLM)])
def test_config_json_matches_the_baseline_fuels(fuel, cfg):
    m = load_fuel(fuel).model
    assert hf_mismatches(m, cfg) == []
    d = model_config_from_hf(cfg)
    assert d.layer_pattern == m.layer_pattern and d.num_experts == m.num_experts and d.mtp_layers == 1


def test_mismatches_are_listed_and_refused(tmp_path):
    m = load_fuel("glm-moe-355b").model
    bad = dict(GLM, partial_rotary_factor=0.5, n_routed_experts=128, use_qk_norm=True)
    msgs = hf_mismatches(m, bad)
    assert {x.split(":")[0] for x in msgs} == {"rotary_fraction", "num_experts", "qk_norm"}
    (tmp_path / "config.json").write_text(json.dumps(bad))
    with pytest.raises(ConfigError, match="disagrees"):
        check_checkpoint_dir(m, str(tmp_path))
    (tmp_path / "config.json").write_text(json.dumps(GLM))
    check_checkpoint_dir(m, str(tmp_path))
    # fewer layers / MTP layers than the checkpoint are allowed, more are not
    assert hf_mismatches(m, dict(GLM, num_hidden_layers=92)) == []
    assert hf_mismatches(m, dict(GLM, num_nextn_predict_layers=0)) == ["mtp_layers: fuel 1 > checkpoint 0"]
    with pytest.raises(ConfigError):
        model_config_from_hf({"model_type": "llama"})


def test_qwen3_moe_and_layer_types():
    q = {"model_type": "qwen3_moe", "hidden_size": 2048, "num_hidden_layers": 48, "num_attention_heads": 32,
         "num_key_value_heads": 4, "head_dim": 128, "rope_theta": 1000000, "rms_norm_eps": 1e-6,
         "vocab_size": 151936, "num_experts": 128, "num_experts_per_tok": 8, "moe_intermediate_size": 768,
         "norm_topk_prob": True, "decoder_sparse_step": 1, "mlp_only_layers": []}
    m = model_config_from_hf(q)
    assert m.num_shared_experts == 0 and m.router == "softmax" and m.qk_norm and m.layer_pattern == ["attention"]
    n = dict(QWEN3_NEXT, layer_types=["linear_attention"] * 3 + ["full_attention"] * 1)
    assert model_config_from_hf(n).layer_pattern == ["deltanet"] * 3 + ["attention"]


def test_fuel_yaml_round_trip(tmp_path):
    doc = fuel_yaml_from_hf(QWEN3_NEXT, "my-next")
    p = tmp_path / "my-next.yaml"
    p.write_text(doc)
    m = load_fuel(str(p)).model
    assert m.name == "my-next" and hf_mismatches(m, QWEN3_NEXT) == []
