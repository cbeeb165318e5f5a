"""The tiny-MoE numerics check: CPU fp32 tiny MoE on NVFP4-dequantized weights vs the
unquantized fp32 model (logits match within tolerance), and the greedy workload."""
import torch

from rocket_b200.config import load_fuel
from rocket_b200.models import ReferenceModel, init_fuel_tensors


def test_tiny_moe_config_matches_baseline():
    c = load_fuel("tiny-moe").model
    assert (c.vocab_size, c.num_layers, c.d_model, c.num_q_heads, c.num_kv_heads, c.head_dim) == (4096, 2, 512, 8, 2, 64)
    assert (c.num_experts, c.moe_intermediate, c.top_k, c.router, c.num_shared_experts) == (16, 256, 2, "softmax", 1)
    assert c.rope_theta == 1e6 and c.norm_eps == 1e-6


def test_nvfp4_logits_match_fp32_model():
    cfg = load_fuel("tiny-moe").model
    t = init_fuel_tensors(cfg, seed=0)
    q = ReferenceModel(cfg, t, quantized=True)
    f = ReferenceModel(cfg, t, quantized=False)
    g = torch.Generator().manual_seed(0)
    for _ in range(2):
        ids = torch.randint(0, cfg.vocab_size, (64,), generator=g)
        a, b = q.logits(ids), f.logits(ids)
        cos = torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), 0).item()
        assert cos > 0.93, cos
        # the NVFP4 model's top logit stays near the fp32 top
        top = b.argmax(-1)
        assert (a.gather(1, top[:, None]) > a.quantile(0.99, dim=-1, keepdim=True)).float().mean() > 0.8


def test_greedy_workload_runs():
    cfg = load_fuel("tiny-moe").model
    t = init_fuel_tensors(cfg, seed=0)
    q = ReferenceModel(cfg, t, quantized=True)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, cfg.vocab_size, (64,), generator=g).tolist() for _ in range(4)]
    outs = [q.generate(p, 32) for p in prompts]
    assert all(len(o) == 32 and all(0 <= x < cfg.vocab_size for x in o) for o in outs)


def test_chunked_gated_delta_rule_equals_the_recurrence():
    """The chunk form (what a tensor-core prefill evaluates) equals the token recurrence,
    per-head and per-channel (KDA) decays, chunk sizes that do and do not divide T."""
    import torch

    from rocket_b200.models.deltanet import chunked_gated_delta_rule

    def recurrence(q, k, v, g, beta, S0):
        S, out = S0.clone(), []
        for t in range(q.shape[0]):
            a = torch.exp(g[t])
            S = (a[:, None] if g.dim() == 2 else a) * S
            u = v[t] - S.t() @ k[t]
            S = S + beta[t] * torch.outer(k[t], u)
            out.append(S.t() @ q[t])
        return torch.stack(out), S

    gen = torch.Generator().manual_seed(0)
    f64 = dict(dtype=torch.float64)
    T, Dk, Dv = 70, 16, 12
    q = torch.randn(T, Dk, generator=gen, **f64)
    k = torch.nn.functional.normalize(torch.randn(T, Dk, generator=gen, **f64), dim=-1)
    v = torch.randn(T, Dv, generator=gen, **f64)
    beta = torch.rand(T, generator=gen, **f64)
    S0 = torch.randn(Dk, Dv, generator=gen, **f64)
    for g in (-torch.rand(T, generator=gen, **f64) * 3, -torch.rand(T, Dk, generator=gen, **f64) * 5):
        o_ref, s_ref = recurrence(q, k, v, g, beta, S0)
        for chunk in (16, 64, 23):
            o, s = chunked_gated_delta_rule(q, k, v, g, beta, S0, chunk)
            assert torch.allclose(o, o_ref, atol=1e-10), (chunk, (o - o_ref).abs().max())
            assert torch.allclose(s, s_ref, atol=1e-10)


def test_attention_biases_enter_the_oracle():
    """attention_bias (GLM-4.5): q/k/v biases are fuel tensors the oracle adds; the
    NVFP4 oracle still tracks the fp32 model, and zero biases change nothing."""
    from rocket_b200.config.schema import model_config
    cfg = model_config("tiny-moe", attention_bias=True)
    t = init_fuel_tensors(cfg, seed=0)
    assert t["layers.0.attn.q_proj.bias"].shape == (cfg.q_dim,) and t["layers.0.attn.k_proj.bias"].shape == (cfg.kv_dim,)
    ids = torch.randint(0, cfg.vocab_size, (32,), generator=torch.Generator().manual_seed(2))
    a = ReferenceModel(cfg, t, quantized=True).logits(ids)
    b = ReferenceModel(cfg, t, quantized=False).logits(ids)
    assert torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), 0).item() > 0.93
    z = dict(t)
    for k in [k for k in t if k.endswith(".bias") and ".attn." in k]:
        z[k] = torch.zeros_like(t[k])
    base = load_fuel("tiny-moe").model
    plain = {k: v for k, v in z.items() if not (k.endswith(".bias") and ".attn." in k)}
    assert torch.allclose(ReferenceModel(cfg, z, quantized=False).logits(ids),
                          ReferenceModel(base, plain, quantized=False).logits(ids))
    assert not torch.allclose(ReferenceModel(cfg, t, quantized=False).logits(ids),
                              ReferenceModel(base, plain, quantized=False).logits(ids), atol=1e-3)
