"""Typed config surface: fuel (model + weights), booster (one GPU node), rocket
(boosters + fabric), engine (parallel degrees, buckets, cache geometry).

The vocabulary is the reference's (``blog/rocket.qmd:9-16``): a *fuel* is a
model plus its weights (``fuels/<id>/fuel.yaml``), a *booster* is one node
(``boosters/<node>.yaml``), a *rocket* is boosters + fabric + handshake
requirements (``boosters/pair.yaml``).  This build adds ``engine.yaml`` for the
per-deployment knobs the reference keeps in CLI flags
(``engines/glm5-moe-nvfp4-2b/src/coding_bench_main.cu:140-176``).

Like the reference's ``load_model_config`` (``src/model_config.h:7-9,92``) the
loader is fail-closed: unknown keys and inconsistent geometry raise.
"""
from __future__ import annotations

import dataclasses
import hashlib
import json
import os
from dataclasses import dataclass, field, fields
from typing import Any

import yaml

_HERE = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.dirname(_HERE)


class ConfigError(ValueError):
    pass


def _from_dict(cls, d: dict[str, Any], where: str):
    names = {f.name: f for f in fields(cls)}
    unknown = set(d) - set(names)
    if unknown:
        raise ConfigError(f"{where}: unknown keys {sorted(unknown)}")
    kwargs = {}
    for k, v in d.items():
        f = names[k]
        sub = _NESTED.get((cls.__name__, k))
        if sub is not None and isinstance(v, dict):
            v = _from_dict(sub, v, f"{where}.{k}")
        kwargs[k] = v
    return cls(**kwargs)


@dataclass
class DeltaNetConfig:
    """Gated DeltaNet linear attention (Qwen3-Next style)."""
    num_qk_heads: int = 16
    num_v_heads: int = 32
    head_dim: int = 128
    conv_kernel: int = 4
    chunk: int = 64
    # "head": one log decay per v head, g = -exp(A_log) * softplus(a + dt_bias) (gated
    # DeltaNet); "channel": one per (head, key channel), g = gate_lower_bound *
    # sigmoid(exp(A_log) * (f + dt_bias)) (Kimi delta attention, KDA)
    gate: str = "head"
    gate_lower_bound: float = -5.0
    out_gate: str = "silu"               # silu | sigmoid: the output gate of the gated RMSNorm


@dataclass
class MlaConfig:
    """Multi-head latent attention without RoPE (NoPE): one 512-wide latent per token is
    cached; queries come through a low-rank (q_lora) projection.  Layers named
    "attention" become MLA layers; head_dim must equal v_head_dim and num_kv_heads 1."""
    q_lora_rank: int = 1536
    kv_lora_rank: int = 512
    qk_nope_head_dim: int = 256
    v_head_dim: int = 256


@dataclass
class SparseAttnConfig:
    """DSA-style sparse attention on the GQA layers: a lightweight indexer scores pools of
    `kpool` tokens (pooled by a per-channel softmax gate) and every query attends only to
    the `top_k` tokens of the best pools plus the open tail."""
    index_heads: int = 32
    index_dim: int = 128
    top_k: int = 2048
    kpool: int = 4


@dataclass
class ModelConfig:
    """Architecture of one fuel.  Covers three model families:
    the tiny CPU-oracle MoE, the GLM-style GQA MoE and the Qwen3-Next hybrid."""
    name: str = "tiny-moe"
    vocab_size: int = 4096
    num_layers: int = 2
    d_model: int = 512
    num_q_heads: int = 8
    num_kv_heads: int = 2
    head_dim: int = 64
    rope_theta: float = 1.0e6
    rotary_fraction: float = 1.0
    norm_eps: float = 1.0e-6
    # first `num_dense_layers` layers use a dense SwiGLU MLP, the rest MoE
    num_dense_layers: int = 0
    dense_intermediate: int = 0
    num_experts: int = 16
    moe_intermediate: int = 256
    top_k: int = 2
    router: str = "softmax"              # softmax | sigmoid
    norm_topk_prob: bool = True
    routed_scaling: float = 1.0
    num_shared_experts: int = 1
    shared_intermediate: int = 256
    shared_expert_gate: bool = False     # Qwen3-Next: sigmoid gate on the shared expert
    # layer pattern: list of "attention" / "deltanet", repeated to num_layers
    layer_pattern: list = field(default_factory=lambda: ["attention"])
    attn_output_gate: bool = False       # Qwen3-Next gated full attention
    qk_norm: bool = False
    attention_bias: bool = False         # q/k/v projection biases (GLM-4.5)
    zero_centered_norm: bool = False     # Gemma/Qwen3-Next (1+w) RMSNorm
    deltanet: DeltaNetConfig | None = None
    mtp_layers: int = 0
    # hidden-tap drafting: the draft head's first pass reads the residual stream after these
    # layers (concatenated, merged by mtp.0.tap_proj [d, n*d]) instead of the last layer's
    # hidden state; empty = the classic MTP head
    mtp_taps: list = field(default_factory=list)
    # manifold-constrained hyper-connections: hc_streams parallel residual streams
    # (0 = one plain residual); Sinkhorn iterations and epsilon of the stream mixing
    sparse_attention: SparseAttnConfig | None = None
    mla: MlaConfig | None = None
    hc_streams: int = 0
    hc_sinkhorn_iters: int = 20
    hc_eps: float = 1.0e-6
    tie_embeddings: bool = False
    init_std: float = 0.02
    weight_format: dict = field(default_factory=lambda: {
        "experts": "nvfp4", "shared": "nvfp4", "dense": "nvfp4", "attention": "bf16",
        "lm_head": "bf16"})

    def layer_kind(self, i: int) -> str:
        return self.layer_pattern[i % len(self.layer_pattern)]

    def is_moe_layer(self, i: int) -> bool:
        return i >= self.num_dense_layers and self.num_experts > 0

    @property
    def q_dim(self) -> int:
        return self.num_q_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_kv_heads * self.head_dim

    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.rotary_fraction)

    def validate(self) -> "ModelConfig":
        if self.num_q_heads % max(self.num_kv_heads, 1):
            raise ConfigError("num_q_heads must be a multiple of num_kv_heads")
        if self.router not in ("softmax", "sigmoid"):
            raise ConfigError(f"router {self.router!r}")
        if self.num_experts and self.top_k > self.num_experts:
            raise ConfigError("top_k > num_experts")
        for kind in self.layer_pattern:
            if kind not in ("attention", "deltanet"):
                raise ConfigError(f"layer kind {kind!r}")
        if "deltanet" in self.layer_pattern and self.deltanet is None:
            raise ConfigError("deltanet layers need a deltanet block")
        if self.deltanet is not None:
            if self.deltanet.gate not in ("head", "channel"):
                raise ConfigError(f"deltanet gate {self.deltanet.gate!r}")
            if self.deltanet.out_gate not in ("silu", "sigmoid"):
                raise ConfigError(f"deltanet out_gate {self.deltanet.out_gate!r}")
        if self.rotary_dim % 2:
            raise ConfigError("rotary dim must be even")
        if self.mla is not None:
            m = self.mla
            if m.kv_lora_rank != 512 or not 1 <= m.qk_nope_head_dim <= 256 or not 1 <= m.v_head_dim <= 512:
                raise ConfigError("mla: kv_lora_rank 512, qk_nope_head_dim <= 256, v_head_dim <= 512")
            if self.head_dim != m.v_head_dim or self.num_kv_heads != 1:
                raise ConfigError("mla: set head_dim = v_head_dim and num_kv_heads = 1")
            if m.q_lora_rank % 64 or m.qk_nope_head_dim % 8 or m.v_head_dim % 8:
                raise ConfigError("mla: q_lora_rank % 64, head dims % 8")
        sa = self.sparse_attention
        if sa is not None:
            if sa.index_dim != 128 or not 1 <= sa.index_heads <= 32 or not 1 <= sa.kpool <= 8 or sa.top_k % sa.kpool:
                raise ConfigError("sparse_attention: index_dim 128, 1..32 index heads, kpool 1..8 dividing top_k")
            if self.mla is None and self.num_q_heads // max(self.num_kv_heads, 1) > (8 if self.head_dim == 256 else 16):
                raise ConfigError("sparse_attention: too many q heads per kv head")
        if self.hc_streams not in (0, 2, 4):
            raise ConfigError("hc_streams must be 0, 2 or 4")
        if self.hc_streams and self.hc_sinkhorn_iters < 1:
            raise ConfigError("hc_sinkhorn_iters must be >= 1")
        for k in (self.d_model, self.moe_intermediate, self.shared_intermediate):
            if k and k % 64:
                raise ConfigError("NVFP4 GEMM dims must be multiples of 64")
        return self

    def fingerprint(self) -> str:
        blob = json.dumps(dataclasses.asdict(self), sort_keys=True).encode()
        return hashlib.sha256(blob).hexdigest()[:16]

    # ---- byte accounting (fail-closed budget checks use these) -----------
    def param_bytes(self, tp: int = 1, ep: int = 1) -> int:
        def nv(n, k):
            return n * k // 2 + n * k // 16
        total = 0
        attn = 0
        for i in range(self.num_layers):
            if self.layer_kind(i) == "attention":
                qd = self.q_dim * (2 if self.attn_output_gate else 1)
                attn += (qd + 2 * self.kv_dim) * self.d_model * 2 + self.q_dim * self.d_model * 2
            else:
                dn = self.deltanet
                kd = dn.num_qk_heads * dn.head_dim
                vd = dn.num_v_heads * dn.head_dim
                attn += (2 * kd + 2 * vd + 2 * dn.num_v_heads) * self.d_model * 2 + vd * self.d_model * 2
            if self.is_moe_layer(i):
                total += self.num_experts * (nv(2 * self.moe_intermediate, self.d_model)
                                             + nv(self.d_model, self.moe_intermediate)) // ep
                total += self.num_shared_experts * (nv(2 * self.shared_intermediate, self.d_model)
                                                    + nv(self.d_model, self.shared_intermediate))
                total += self.num_experts * self.d_model * 2
            else:
                total += nv(2 * self.dense_intermediate, self.d_model) + nv(self.d_model, self.dense_intermediate)
        total += attn // tp
        total += 2 * self.vocab_size * self.d_model * 2 // tp
        return total


@dataclass
class FuelConfig:
    id: str = "tiny-moe"
    chemistry: str = ""
    status: str = "synthetic"
    model: ModelConfig = field(default_factory=ModelConfig)
    notes: str = ""


@dataclass
class BoosterConfig:
    """One GPU node.  Facts the mount probe checks at ignition."""
    id: str = "b200x8"
    gpus: int = 8
    gpu_name: str = "NVIDIA B200"
    sm_count: int = 148
    hbm_gib: float = 179.0
    hbm_gbs_measured: float = 6548.8
    bf16_tflops_measured: float = 1631.7
    nvlink_gbs_per_dir: float = 770.0
    smem_per_block_optin: int = 232448
    compute_capability: str = "10.0"


@dataclass
class RocketConfig:
    id: str = "b200x8-nvswitch"
    boosters: list = field(default_factory=lambda: ["b200x8"])
    arrangement: str = "single-node"
    fabric: dict = field(default_factory=lambda: {"kind": "nvswitch", "nccl": True, "p2p": True})
    handshake_requirements: dict = field(default_factory=dict)


@dataclass
class EngineConfig:
    """Per-deployment engine knobs."""
    tp: int = 1
    ep: int = 1
    max_batch: int = 64
    batch_buckets: list = field(default_factory=lambda: [1, 2, 4, 8, 16, 32, 64, 128, 256])
    page_size: int = 64
    kv_dtype: str = "bf16"              # bf16 | fp8
    max_seq_len: int = 4096
    num_pages: int = 0                  # 0 = derive from memory budget
    kv_memory_fraction: float = 0.9
    prefill_chunk: int = 8192           # token budget per scheduler step
    cuda_graphs: bool = True
    spec_tokens: int = 0                # MTP draft tokens per step (0 = off)
    draft_source: str = "mtp"           # '+'-joined priority list: mtp | prompt_lookup | history | file
    spec_depth: str = "fixed"           # fixed: spec_tokens drafts every step | adaptive: engine/depth.py
    draft_file: str = ""                # reference generation for the 'file' source
    collectives: str = "fused"          # multi-GPU decode: fused (in-kernel all-reduce / combine) | sp | nccl
    expert_cache_slots: int = 0         # > 0: routed experts stream from host memory into this many slots per layer
    prefix_cache: bool = True
    prefix_store_dir: str = ""
    seed: int = 0


_NESTED = {
    ("ModelConfig", "deltanet"): DeltaNetConfig,
    ("ModelConfig", "sparse_attention"): SparseAttnConfig,
    ("ModelConfig", "mla"): MlaConfig,
    ("FuelConfig", "model"): ModelConfig,
}


def _load_yaml(path: str) -> dict:
    with open(path) as f:
        d = yaml.safe_load(f) or {}
    if not isinstance(d, dict):
        raise ConfigError(f"{path}: top level must be a mapping")
    return d


def load_fuel(name_or_path: str) -> FuelConfig:
    path = name_or_path
    if not os.path.exists(path):
        path = os.path.join(PKG_ROOT, "fuels", f"{name_or_path}.yaml")
    if not os.path.exists(path):
        raise ConfigError(f"no fuel {name_or_path!r}")
    fuel = _from_dict(FuelConfig, _load_yaml(path), os.path.basename(path))
    fuel.model.validate()
    return fuel


def load_booster(name_or_path: str) -> BoosterConfig:
    path = name_or_path
    if not os.path.exists(path):
        path = os.path.join(PKG_ROOT, "boosters", f"{name_or_path}.yaml")
    return _from_dict(BoosterConfig, _load_yaml(path), os.path.basename(path))


def load_rocket(name_or_path: str) -> RocketConfig:
    path = name_or_path
    if not os.path.exists(path):
        path = os.path.join(PKG_ROOT, "boosters", f"{name_or_path}.yaml")
    return _from_dict(RocketConfig, _load_yaml(path), os.path.basename(path))


def load_engine(path_or_dict, **overrides) -> EngineConfig:
    """Engine knobs from a YAML file, a preset name under rocket_b200/engines, or a dict;
    keyword overrides (None = keep) win over the file."""
    if isinstance(path_or_dict, str) and path_or_dict and not os.path.exists(path_or_dict):
        preset = os.path.join(PKG_ROOT, "engines", f"{path_or_dict}.yaml")
        if not os.path.exists(preset):
            raise ConfigError(f"no engine config {path_or_dict!r}")
        path_or_dict = preset
    d = dict(path_or_dict) if isinstance(path_or_dict, dict) else (_load_yaml(path_or_dict) if path_or_dict else {})
    d.update({k: v for k, v in overrides.items() if v is not None})
    e = _from_dict(EngineConfig, d, "engine")
    if e.page_size not in (16, 32, 64, 128):
        raise ConfigError("page_size must be 16/32/64/128")
    if e.kv_dtype not in ("bf16", "fp8"):
        raise ConfigError("kv_dtype must be bf16 or fp8")
    if e.expert_cache_slots < 0:
        raise ConfigError("expert_cache_slots must be >= 0 (0 = every routed expert resident)")
    return e


def model_config(name: str, **overrides) -> ModelConfig:
    m = load_fuel(name).model
    return dataclasses.replace(m, **overrides).validate() if overrides else m
