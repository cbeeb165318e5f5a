"""Fuel-format weights, random initialisation, and conversion to the engine layout.

Fuel format (what a checkpoint on disk holds; names are this framework's):

    embed.weight                         [V, d]    bf16
    layers.{i}.attn_norm.weight          [d]
    layers.{i}.attn.{q,k,v,o}_proj.*     bf16 ``.weight`` or an NVFP4 triplet
                                         (``.weight`` u8 [N,K/2], ``.weight_scale`` u8 e4m3 [N,K/16],
                                         ``.weight_scale_2`` f32 scalar); q_proj of a gated-attention
                                         layer has 2*Hq*D rows: [q | gate]; ``.bias`` [rows] bf16
                                         on q/k/v when attention_bias
    layers.{i}.attn.{q,k}_norm.weight    [D]            (qk_norm)
    layers.{i}.mlp_norm.weight           [d]
    layers.{i}.mlp.{gate,up,down}_proj.* NVFP4          (dense layers)
    layers.{i}.moe.router.weight         [E, d] bf16;   router.bias [E] f32 (sigmoid routing)
    layers.{i}.moe.experts.{e}.{gate,up,down}_proj.*    NVFP4
    layers.{i}.moe.shared.{gate,up,down}_proj.*         NVFP4
    layers.{i}.moe.shared_gate.weight    [1, d] bf16    (shared_expert_gate)
    layers.{i}.dn.*                      gated DeltaNet (see deltanet.py)
    final_norm.weight, lm_head.weight
    mtp.{j}.{enorm,hnorm}.weight         [d]  multi-token-prediction head j
    mtp.{j}.eh_proj.weight               [d, 2d] bf16 over [enorm(embed(next token)) | hnorm(hidden)]
    mtp.{j}.layer.*                      one attention + MoE (or dense) block, named like layers.{i}
    mtp.{j}.norm.weight                  [d]  norm before the shared lm_head
    mtp.0.tap_proj.weight                [d, n*d] bf16: merges the tapped hidden states (mtp_taps)

The NVFP4 triplet is the reference's on-disk layout
(engines/glm5-moe-nvfp4-2b/src/nvfp4.h:4-11).

Engine layout: fused ``w13`` with gate/up rows interleaved in 64-row halves of
every 128-row tile (the GEMM's SwiGLU epilogue pairs row r with row r+64),
scale factors in tcgen05 atoms, per-row tensor scales; experts of a layer are
stacked with the shared experts appended.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from ..config import ModelConfig
from ..fuel import nvfp4 as nv


def _fmt(cfg: ModelConfig, part: str) -> str:
    return cfg.weight_format.get(part, "bf16")


def _gen(seed: int, device="cpu"):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _randn(shape, std, g, device="cpu"):
    return torch.randn(*shape, generator=g, device=device) * std


def quantize_fp8_rows(w: torch.Tensor):
    """e4m3 weight rows with per-row fp32 scales amax / 448 (the FP8-row fuel format)."""
    w = w.float()
    amax = w.abs().amax(dim=1)
    scale = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    return (w / scale.unsqueeze(1)).clamp(-448, 448).to(torch.float8_e4m3fn), scale


def _put_linear(t: dict, name: str, w: torch.Tensor, fmt: str):
    if fmt == "fp8":
        q, sc = quantize_fp8_rows(w)
        t[name + ".weight"] = q
        t[name + ".weight_scale"] = sc
    elif fmt == "nvfp4":
        p, s, gs = nv.quantize_nvfp4(w)
        t[name + ".weight"] = p
        t[name + ".weight_scale"] = s
        t[name + ".weight_scale_2"] = torch.tensor(gs, dtype=torch.float32)
    else:
        t[name + ".weight"] = w.bfloat16()


def init_fuel_tensors(cfg: ModelConfig, seed: int = 0) -> dict:
    """Random-init N(0, init_std) fuel tensors on the CPU (small models only).

    Returns fp32 masters too under ``master.*`` keys so tests can build the
    unquantized fp32 model (the tiny-MoE numerics comparison).
    """
    g = _gen(seed)
    std = cfg.init_std
    d = cfg.d_model
    t: dict[str, torch.Tensor] = {}
    m: dict[str, torch.Tensor] = {}

    def lin(name, n, k, part):
        w = _randn((n, k), std, g)
        m[name] = w
        _put_linear(t, name, w, _fmt(cfg, part))

    t["embed.weight"] = _randn((cfg.vocab_size, d), std, g).bfloat16()
    m["embed"] = t["embed.weight"].float()
    one = lambda n: (torch.zeros(n) if cfg.zero_centered_norm else torch.ones(n)).bfloat16()
    def hyper(pre):
        # mHC mixing of hc residual streams around each sub-layer: W_mix [2hc+hc^2, hc*d],
        # bias [2hc+hc^2] (fp32), scales [3] (pre / post / comb, fp32)
        hc = cfg.hc_streams
        nm = 2 * hc + hc * hc
        for site in ("hc_attn", "hc_mlp"):
            t[f"{pre}.{site}.fn"] = _randn((nm, hc * d), std, g).bfloat16()
            t[f"{pre}.{site}.base"] = _randn((nm,), 0.5, g)
            t[f"{pre}.{site}.scale"] = torch.ones(3)

    def block(pre, kind, moe, hc=False):
        t[f"{pre}.attn_norm.weight"] = one(d)
        t[f"{pre}.mlp_norm.weight"] = one(d)
        if hc:
            hyper(pre)
        if kind == "attention" and cfg.mla is not None:
            ml, H = cfg.mla, cfg.num_q_heads
            lin(f"{pre}.attn.q_a_proj", ml.q_lora_rank, d, "attention")
            t[f"{pre}.attn.q_a_norm.weight"] = torch.ones(ml.q_lora_rank).bfloat16()
            lin(f"{pre}.attn.q_b_proj", H * ml.qk_nope_head_dim, ml.q_lora_rank, "attention")
            lin(f"{pre}.attn.kv_a_proj", ml.kv_lora_rank, d, "attention")
            t[f"{pre}.attn.kv_a_norm.weight"] = torch.ones(ml.kv_lora_rank).bfloat16()
            lin(f"{pre}.attn.kv_b_proj", H * (ml.qk_nope_head_dim + ml.v_head_dim), ml.kv_lora_rank, "attention")
            lin(f"{pre}.attn.o_proj", d, H * ml.v_head_dim, "attention")
        elif kind == "attention":
            qrows = cfg.q_dim * (2 if cfg.attn_output_gate else 1)
            lin(f"{pre}.attn.q_proj", qrows, d, "attention")
            lin(f"{pre}.attn.k_proj", cfg.kv_dim, d, "attention")
            lin(f"{pre}.attn.v_proj", cfg.kv_dim, d, "attention")
            lin(f"{pre}.attn.o_proj", d, cfg.q_dim, "attention")
            if cfg.attention_bias:
                for nm, n in (("q_proj", qrows), ("k_proj", cfg.kv_dim), ("v_proj", cfg.kv_dim)):
                    t[f"{pre}.attn.{nm}.bias"] = _randn((n,), 0.5, g).bfloat16()
            if cfg.qk_norm and cfg.mla is None:
                t[f"{pre}.attn.q_norm.weight"] = one(cfg.head_dim)
                t[f"{pre}.attn.k_norm.weight"] = one(cfg.head_dim)
        if kind == "attention":
            sa = cfg.sparse_attention
            if sa is not None:
                ip = f"{pre}.attn.indexer"
                Hi, Di = sa.index_heads, sa.index_dim
                lin(f"{ip}.wq", Hi * Di, d, "indexer")
                lin(f"{ip}.wk", Di, d, "indexer")
                lin(f"{ip}.wgate", Di, d, "indexer")
                lin(f"{ip}.wproj", Hi, d, "indexer")
                t[f"{ip}.k_norm.weight"] = torch.ones(Di)
                t[f"{ip}.k_norm.bias"] = torch.zeros(Di)
                t[f"{ip}.ape"] = _randn((sa.kpool, Di), 0.5, g)
        else:
            from .deltanet import init_deltanet_tensors
            init_deltanet_tensors(cfg, pre, t, m, g, lin, one)
        if moe:
            E = cfg.num_experts
            t[f"{pre}.moe.router.weight"] = _randn((E, d), std, g).bfloat16()
            m[f"{pre}.moe.router"] = t[f"{pre}.moe.router.weight"].float()
            if cfg.router == "sigmoid":
                t[f"{pre}.moe.router.bias"] = torch.zeros(E, dtype=torch.float32)
            for e in range(E):
                lin(f"{pre}.moe.experts.{e}.gate_proj", cfg.moe_intermediate, d, "experts")
                lin(f"{pre}.moe.experts.{e}.up_proj", cfg.moe_intermediate, d, "experts")
                lin(f"{pre}.moe.experts.{e}.down_proj", d, cfg.moe_intermediate, "experts")
            for s in range(cfg.num_shared_experts):
                sn = f"{pre}.moe.shared" if cfg.num_shared_experts == 1 else f"{pre}.moe.shared.{s}"
                lin(f"{sn}.gate_proj", cfg.shared_intermediate, d, "shared")
                lin(f"{sn}.up_proj", cfg.shared_intermediate, d, "shared")
                lin(f"{sn}.down_proj", d, cfg.shared_intermediate, "shared")
            if cfg.shared_expert_gate:
                t[f"{pre}.moe.shared_gate.weight"] = _randn((1, d), std, g).bfloat16()
                m[f"{pre}.moe.shared_gate"] = t[f"{pre}.moe.shared_gate.weight"].float()
        else:
            lin(f"{pre}.mlp.gate_proj", cfg.dense_intermediate, d, "dense")
            lin(f"{pre}.mlp.up_proj", cfg.dense_intermediate, d, "dense")
            lin(f"{pre}.mlp.down_proj", d, cfg.dense_intermediate, "dense")
    for i in range(cfg.num_layers):
        block(f"layers.{i}", cfg.layer_kind(i), cfg.is_moe_layer(i), hc=cfg.hc_streams > 0)
    t["final_norm.weight"] = one(d)
    lin("lm_head", cfg.vocab_size, d, "lm_head")
    # multi-token-prediction heads (after every other tensor, so they do not shift the
    # random streams of the base model)
    for j in range(cfg.mtp_layers):
        pre = f"mtp.{j}"
        t[f"{pre}.enorm.weight"] = one(d)
        t[f"{pre}.hnorm.weight"] = one(d)
        lin(f"{pre}.eh_proj", d, 2 * d, "eh_proj")  # bf16 unless weight_format names eh_proj
        block(f"{pre}.layer", "attention", cfg.num_experts > 0)
        t[f"{pre}.norm.weight"] = one(d)
        if j == 0 and cfg.mtp_taps:
            lin(f"{pre}.tap_proj", d, len(cfg.mtp_taps) * d, "tap_proj")  # bf16
    t.update({"master." + k: v for k, v in m.items()})
    return t


def dequant(t: dict, name: str) -> torch.Tensor:
    """fp32 value of linear `name` (dequantized when stored as NVFP4 or FP8-row)."""
    if t[name + ".weight"].dtype == torch.float8_e4m3fn:
        return t[name + ".weight"].float() * t[name + ".weight_scale"].float().unsqueeze(1)
    if name + ".weight_scale" in t:
        return nv.dequantize_nvfp4(t[name + ".weight"], t[name + ".weight_scale"],
                                   float(t[name + ".weight_scale_2"]))
    return t[name + ".weight"].float()


# ---------------------------------------------------------------- engine layout
def interleave_w13(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """[I, ...] gate/up rows -> [2I, ...] with rows [64 gate | 64 up] per 128-row tile."""
    I = gate.shape[0]
    assert I % 64 == 0, "intermediate must be a multiple of 64"
    gt = gate.reshape(I // 64, 64, *gate.shape[1:])
    ut = up.reshape(I // 64, 64, *up.shape[1:])
    return torch.stack([gt, ut], 1).reshape(2 * I, *gate.shape[1:])


@dataclass
class NvTriplet:
    packed: torch.Tensor      # [N, K/2] u8
    sf: torch.Tensor          # [N, K/16] u8 (linear)
    gscale: torch.Tensor      # [N] f32 per-row tensor scale


def triplet_of(t: dict, name: str) -> NvTriplet:
    p = t[name + ".weight"]
    return NvTriplet(p, t[name + ".weight_scale"],
                     torch.full((p.shape[0],), float(t[name + ".weight_scale_2"]), dtype=torch.float32))


def fuse_w13(gate: NvTriplet, up: NvTriplet) -> NvTriplet:
    return NvTriplet(interleave_w13(gate.packed, up.packed), interleave_w13(gate.sf, up.sf),
                     interleave_w13(gate.gscale, up.gscale))


def stack_nvfp4(trips: list[NvTriplet], device):
    """Stack per-expert triplets into one engine NvFp4Weight."""
    from ..ops import NvFp4Weight
    n = trips[0].packed.shape[0]
    k = trips[0].packed.shape[1] * 2
    packed = torch.cat([x.packed for x in trips], 0).to(device)
    sf = torch.cat([nv.swizzle_sf(x.sf) for x in trips], 0).to(device)
    g = torch.cat([x.gscale for x in trips], 0).to(device)
    return NvFp4Weight(packed, sf, g, n, k, len(trips))


def empty_nvfp4(n: int, k: int, experts: int, device):
    """Uninitialised stacked NVFP4 weight (filled by the expert-slab loader)."""
    from ..ops import NvFp4Weight
    packed = torch.empty(experts * n, k // 2, dtype=torch.uint8, device=device)
    sf = torch.empty(experts * nv.sf_swizzled_bytes(n, k), dtype=torch.uint8, device=device)
    g = torch.empty(experts * n, dtype=torch.float32, device=device)
    return NvFp4Weight(packed, sf, g, n, k, experts)


def pad_rows(w: torch.Tensor, mult: int = 128) -> torch.Tensor:
    n = w.shape[0]
    np_ = (n + mult - 1) // mult * mult
    if np_ == n:
        return w
    out = torch.zeros(np_, *w.shape[1:], dtype=w.dtype)
    out[:n] = w
    return out


def set_expert_tail(w, tail):
    """Overwrite the last tail.num_experts experts of the stacked NVFP4 weight w with tail's."""
    n_t = tail.num_experts
    e0 = w.num_experts - n_t
    pk, sf, gs = w.packed.numel() // w.num_experts, w.sf.numel() // w.num_experts, w.gscale.numel() // w.num_experts
    w.packed.view(-1)[e0 * pk:].copy_(tail.packed.view(-1))
    w.sf.view(-1)[e0 * sf:].copy_(tail.sf.view(-1))
    w.gscale.view(-1)[e0 * gs:].copy_(tail.gscale.view(-1))


def random_nvfp4_on_device(shape_nk, experts: int, std: float, gen: torch.Generator, device,
                           fuse_swiglu: bool = False):
    """Random N(0,std) NVFP4 weights generated and quantized on the GPU.

    One tensor scale per expert (per gate/up half when `fuse_swiglu`), the
    ModelOpt amax/(448*6) rule.  Returns an engine ``NvFp4Weight``.
    """
    from .. import ops
    n, k = shape_nk
    packed = torch.empty(experts * n, k // 2, dtype=torch.uint8, device=device)
    sf = torch.empty(experts * n // 128 * (k // 64) * 512, dtype=torch.uint8, device=device)
    gs_rows = torch.empty(experts * n, dtype=torch.float32, device=device)
    chunk = max(1, min(experts, (1 << 31) // (n * k * 2)))
    for e0 in range(0, experts, chunk):
        e1 = min(experts, e0 + chunk)
        w = torch.randn((e1 - e0) * n, k, generator=gen, device=device, dtype=torch.bfloat16) * std
        groups = (e1 - e0) * (2 if fuse_swiglu else 1)
        # tensors: each expert (or each gate/up half) is one NVFP4 tensor
        if fuse_swiglu:
            # rows of tensor j in interleaved w13: tile t rows [64 gate | 64 up]
            wv = w.view(e1 - e0, n // 128, 2, 64, k)
            amax = wv.abs().amax(dim=(1, 3, 4)).float()            # [E, 2]
            g = (amax / 2688.0).clamp_min(1e-12)
            row_g = g.view(e1 - e0, 1, 2, 1).expand(e1 - e0, n // 128, 2, 64).reshape(-1).contiguous()
        else:
            amax = w.view(e1 - e0, -1).abs().amax(dim=1).float()
            g = (amax / 2688.0).clamp_min(1e-12)
            row_g = g.repeat_interleave(n).contiguous()
        r0, r1 = e0 * n, e1 * n
        sf_lo = r0 // 128 * (k // 64) * 512
        sf_hi = r1 // 128 * (k // 64) * 512
        ops.quantize_weight_rows(w, row_g, 1, packed[r0:r1], sf[sf_lo:sf_hi])
        gs_rows[r0:r1] = row_g
        del w
    return ops.NvFp4Weight(packed, sf, gs_rows, n, k, experts)
