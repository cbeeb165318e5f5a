"""CPU fp32 oracle of the model families (the "offline parity oracle").

Written from the model arithmetic (RMSNorm, RoPE rotate-half, GQA causal
softmax attention, softmax/sigmoid top-k routing, SwiGLU experts, shared
expert), independent of the GPU kernels it is used to check -- the same rule
as the reference's CPU tests (engines/glm5-moe-nvfp4-2b/tests/test_kernels.cu:1-3).

``ReferenceModel(cfg, tensors, quantized=True)`` runs on the NVFP4-dequantized
weights; ``quantized=False`` on the fp32 masters (the tiny-MoE numerics check
compares the two).  ``emulate_gpu=True`` additionally applies the GPU path's numerics:
per-row NVFP4 quantization of the activations entering NVFP4 GEMMs and bf16
rounding where the GPU stores bf16, so GPU-vs-oracle tolerances can be tight.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from ..config import ModelConfig
from ..fuel import nvfp4 as nv
from .weights import dequant


def _bf(x):
    return x.bfloat16().float()


def _qact(x):
    """NVFP4 round trip of activation rows (per-row tensor scale), as the GPU does."""
    shp = x.shape
    x2 = x.reshape(-1, shp[-1])
    p, s, g = nv.quantize_rows_nvfp4_reference(x2)
    return (nv.dequantize_nvfp4(p, s, 1.0) * g.unsqueeze(1)).reshape(shp)


def _qact8(x):
    """Per-row e4m3 round trip of activation rows (scale amax / 448), as the FP8 GEMM path does."""
    shp = x.shape
    x2 = x.reshape(-1, shp[-1]).float()
    amax = x2.abs().amax(dim=1, keepdim=True)
    s = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    return ((x2 / s).to(torch.float8_e4m3fn).float() * s).reshape(shp)


class ReferenceModel:
    def __init__(self, cfg: ModelConfig, tensors: dict, quantized: bool = True, emulate_gpu: bool = False):
        self.cfg = cfg
        self.t = tensors
        self.quantized = quantized
        self.emu = emulate_gpu
        self._w = {}

    # ---------------------------------------------------------------- weights
    def W(self, name):
        if name not in self._w:
            if self.quantized:
                self._w[name] = dequant(self.t, name)
            else:
                self._w[name] = self.t["master." + name].float()
        return self._w[name]

    def is_fp8(self, name):
        return self.quantized and self.t[name + ".weight"].dtype == torch.float8_e4m3fn

    def is_nv(self, name):
        return self.quantized and (name + ".weight_scale") in self.t and not self.is_fp8(name)

    def _act_site(self, name):
        """(layer prefix, site, which rows) of linear `name`'s NVFP4 input in the GPU's taps."""
        for suf, site in ((".attn.q_proj", "attn_in"), (".attn.k_proj", "attn_in"), (".attn.v_proj", "attn_in"),
                          (".attn.o_proj", "attn_out"), (".mlp.gate_proj", "dense_in"), (".mlp.up_proj", "dense_in"),
                          (".mlp.down_proj", "dense_h")):
            if name.endswith(suf):
                return name[: -len(suf)], site
        if ".moe." in name:
            lpre = name.split(".moe.")[0]
            return lpre, ("moe_h" if name.endswith(".down_proj") else "moe_in")
        return None, None

    def lin(self, x, name):
        w = self.W(name)
        ov = getattr(self, "act_override", None)
        if self.emu and ov is not None and self.is_nv(name):
            # the GPU's own dequantized NVFP4 codes for this input (numerics tests)
            lpre, site = self._act_site(name)
            a = ov.get((lpre, site))
            if a is not None:
                rows, slot = getattr(self, "_moe_rows", (None, None))
                if site == "moe_h":
                    x = a[rows, slot]
                elif site == "moe_in":
                    x = a[rows]
                else:
                    x = a
                y = x @ w.t()
                b = self.t.get(name + ".bias")
                return y + b.float() if b is not None else y
        if self.emu:
            x = _qact(x) if self.is_nv(name) else (_qact8(_bf(x)) if self.is_fp8(name) else _bf(x))
        y = x @ w.t()
        b = self.t.get(name + ".bias")
        if b is not None:
            y = (_bf(y) if self.emu else y) + b.float()  # the engine adds the bias to the stored bf16 output
        return y

    def norm(self, x, w, eps=None):
        eps = self.cfg.norm_eps if eps is None else eps
        w = w.float()
        if self.cfg.zero_centered_norm:
            w = w + 1.0
        y = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w
        return _bf(y) if self.emu else y

    # ---------------------------------------------------------------- blocks
    def rope(self, x, pos):
        # x [T, H, D]; rotate-half over the first rotary_dim dims
        rot = self.cfg.rotary_dim
        i = torch.arange(rot // 2, dtype=torch.float64)
        inv = (1.0 / (self.cfg.rope_theta ** (2 * i / rot))).float()
        ang = pos.float().unsqueeze(1) * inv.unsqueeze(0)
        cos, sin = torch.cos(ang).unsqueeze(1), torch.sin(ang).unsqueeze(1)
        a, b = x[..., : rot // 2], x[..., rot // 2: rot]
        return torch.cat([a * cos - b * sin, b * cos + a * sin, x[..., rot:]], -1)

    def mla_attention(self, lpre, x):
        """MLA (NoPE) in the non-absorbed form: per-head keys / values up-projected from the
        normalized latent; the GPU runs the absorbed form (same math in exact arithmetic)."""
        c, ml = self.cfg, self.cfg.mla
        T, H, nope, v = x.shape[0], c.num_q_heads, ml.qk_nope_head_dim, ml.v_head_dim
        pre = f"{lpre}.attn"

        def rms(y, w):
            return y * torch.rsqrt(y.pow(2).mean(-1, keepdim=True) + c.norm_eps) * w.float()

        qa = self.lin(x, f"{pre}.q_a_proj")
        if self.emu:
            qa = _bf(qa)
        qa = rms(qa, self.t[f"{pre}.q_a_norm.weight"])
        if self.emu:
            qa = _bf(qa)
        q = self.lin(qa, f"{pre}.q_b_proj").view(T, H, nope)
        lat = self.lin(x, f"{pre}.kv_a_proj")
        if self.emu:
            q, lat = _bf(q), _bf(lat)
        lat = rms(lat, self.t[f"{pre}.kv_a_norm.weight"])
        if self.emu:
            lat = _bf(lat)
        kvb = self.W(f"{pre}.kv_b_proj")
        if self.emu:
            kvb = _bf(kvb)
        kvb = kvb.view(H, nope + v, ml.kv_lora_rank)
        k = torch.einsum("tc,hdc->thd", lat, kvb[:, :nope])
        vv = torch.einsum("tc,hdc->thd", lat, kvb[:, nope:])
        s = torch.einsum("qhd,khd->hqk", q, k) / math.sqrt(nope)
        mask = torch.ones(T, T, dtype=torch.bool).tril()
        if c.sparse_attention is not None:
            mask = self.dsa_mask(f"{pre}.indexer", x)
        s = s.masked_fill(~mask, float("-inf"))
        o = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), vv).reshape(T, H * v)
        if self.emu:
            o = _bf(o)
        return self.lin(o, f"{pre}.o_proj")

    def attention(self, lpre, x, pos):
        c = self.cfg
        if c.mla is not None:
            return self.mla_attention(lpre, x)
        T = x.shape[0]
        pre = f"{lpre}.attn"
        q_all = self.lin(x, f"{pre}.q_proj")
        k = self.lin(x, f"{pre}.k_proj").view(T, c.num_kv_heads, c.head_dim)
        v = self.lin(x, f"{pre}.v_proj").view(T, c.num_kv_heads, c.head_dim)
        if c.attn_output_gate:
            q = q_all[:, : c.q_dim].view(T, c.num_q_heads, c.head_dim)
            gate = q_all[:, c.q_dim:].view(T, c.num_q_heads, c.head_dim)
        else:
            q, gate = q_all.view(T, c.num_q_heads, c.head_dim), None
        if self.emu:
            q, k, v = _bf(q), _bf(k), _bf(v)
            gate = _bf(gate) if gate is not None else None
        if c.qk_norm:
            q = self.norm(q, self.t[f"{pre}.q_norm.weight"])
            k = self.norm(k, self.t[f"{pre}.k_norm.weight"])
        q = self.rope(q, pos)
        k = self.rope(k, pos)
        if self.emu:
            q, k = _bf(q), _bf(k)
        G = c.num_q_heads // c.num_kv_heads
        kk = k.repeat_interleave(G, 1)
        vv = v.repeat_interleave(G, 1)
        s = torch.einsum("qhd,khd->hqk", q, kk) / math.sqrt(c.head_dim)
        mask = torch.ones(T, T, dtype=torch.bool).tril()
        if c.sparse_attention is not None:
            mask = self.dsa_mask(f"{pre}.indexer", x)
        s = s.masked_fill(~mask, float("-inf"))
        o = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), vv)
        if gate is not None:
            o = o * torch.sigmoid(gate)
        o = o.reshape(T, c.q_dim)
        if self.emu:
            o = _bf(o)
        return self.lin(o, f"{pre}.o_proj")

    def dsa_mask(self, ip, x):
        """[T, T] mask of the tokens each row attends to under DSA: the top_k / kpool best
        complete pools (ties to the lower pool index) expanded to tokens, plus the open tail."""
        sa = self.cfg.sparse_attention
        T = x.shape[0]
        Hi, Di, kp = sa.index_heads, sa.index_dim, sa.kpool
        iq = self.lin(x, f"{ip}.wq")
        ik = self.lin(x, f"{ip}.wk")
        ig = self.lin(x, f"{ip}.wgate")
        iw = self.lin(x, f"{ip}.wproj")
        if self.emu:
            iq, ik, ig, iw = _bf(iq), _bf(ik), _bf(ig), _bf(iw)
        mu = ik.mean(-1, keepdim=True)
        var = (ik - mu).pow(2).mean(-1, keepdim=True)
        ik = (ik - mu) * torch.rsqrt(var + 1e-6) * self.t[f"{ip}.k_norm.weight"].float() + \
            self.t[f"{ip}.k_norm.bias"].float()
        if self.emu:
            ik = _bf(ik)
        iq = iq.view(T, Hi, Di)
        ape = self.t[f"{ip}.ape"].float()
        want = sa.top_k // kp
        mask = torch.zeros(T, T, dtype=torch.bool)
        for r in range(T):
            n_tok = r + 1
            P = n_tok // kp
            pools = list(range(P))
            if P > want:
                g = ig[:P * kp].view(P, kp, Di) + ape.view(1, kp, Di)
                pk = (torch.softmax(g, 1) * ik[:P * kp].view(P, kp, Di)).sum(1)
                sc = (iw[r].view(Hi, 1) * torch.relu(iq[r] @ pk.t() / math.sqrt(Di))).sum(0)
                pools = sorted(range(P), key=lambda p: (-float(sc[p]), p))[:want]
            for p in pools:
                mask[r, p * kp:(p + 1) * kp] = True
            mask[r, P * kp:n_tok] = True
        return mask

    def swiglu(self, x, pre):
        g = self.lin(x, f"{pre}.gate_proj")
        u = self.lin(x, f"{pre}.up_proj")
        h = F.silu(g) * u
        if self.emu:
            h = _bf(h)
        y = self.lin(h, f"{pre}.down_proj")
        return _bf(y) if self.emu else y

    def moe(self, lpre, x):
        c = self.cfg
        pre = f"{lpre}.moe"
        logits = _bf(x) @ self.W(f"{pre}.router").t() if self.emu else x @ self.W(f"{pre}.router").t()
        # route_override[lpre]: expert choices [T, top_k] to use instead of this top-k (a
        # comparison that must not count near-tie routing flips as a difference); the
        # weights still come from these probabilities
        forced = (getattr(self, "route_override", None) or {}).get(lpre)
        if c.router == "softmax":
            p = torch.softmax(logits, -1)
            sel = torch.topk(p, c.top_k, -1).indices if forced is None else forced
            w = torch.gather(p, 1, sel)
        else:
            s = torch.sigmoid(logits)
            bias = self.t.get(f"{pre}.router.bias", torch.zeros(c.num_experts))
            sel = torch.topk(s + bias, c.top_k, -1).indices if forced is None else forced
            w = torch.gather(s, 1, sel)
        if c.norm_topk_prob:
            w = w / w.sum(-1, keepdim=True)
        w = w * c.routed_scaling
        out = torch.zeros_like(x)
        for e in sel.unique().tolist():
            rows, slot = (sel == e).nonzero(as_tuple=True)
            self._moe_rows = (rows, slot)  # which tokens / routing slots (activation overrides)
            out[rows] += w[rows, slot].unsqueeze(1) * self.swiglu(x[rows], f"{pre}.experts.{e}")
        allr = torch.arange(x.shape[0])
        self._moe_rows = (allr, torch.full_like(allr, c.top_k))  # the shared expert's slot
        sh = self.swiglu(x, f"{pre}.shared")
        self._moe_rows = (None, None)
        if c.shared_expert_gate:
            gl = (_bf(x) if self.emu else x) @ self.W(f"{pre}.shared_gate").t()
            sh = sh * torch.sigmoid(gl)
        return out + sh

    def layer(self, i, x, pos):
        c = self.cfg
        return self.block(f"layers.{i}", c.layer_kind(i), c.is_moe_layer(i), x, pos)

    # ---------------------------------------------------------------- hyper-connections
    def hc_pre(self, site, S):
        """S [T, hc, d] streams -> (sub-layer input [T, d], post [T, hc], comb [T, hc, hc])."""
        c = self.cfg
        T, hc, d = S.shape
        flat = S.reshape(T, hc * d)
        inv = torch.rsqrt(flat.pow(2).mean(-1, keepdim=True) + c.norm_eps)
        mix = (flat @ self.t[f"{site}.fn"].float().t()) * inv
        b = self.t[f"{site}.base"].float()
        sc = self.t[f"{site}.scale"].float()
        eps = c.hc_eps
        pre = torch.sigmoid(mix[:, :hc] * sc[0] + b[:hc]) + eps
        post = 2 * torch.sigmoid(mix[:, hc:2 * hc] * sc[1] + b[hc:2 * hc])
        cm = torch.softmax(mix[:, 2 * hc:].view(T, hc, hc) * sc[2] + b[2 * hc:].view(hc, hc), -1) + eps
        cm = cm / (cm.sum(1, keepdim=True) + eps)            # columns
        for _ in range(c.hc_sinkhorn_iters - 1):
            cm = cm / (cm.sum(2, keepdim=True) + eps)        # rows
            cm = cm / (cm.sum(1, keepdim=True) + eps)        # columns
        x = (pre.unsqueeze(-1) * S).sum(1)
        return (_bf(x) if self.emu else x), post, cm

    def hc_post(self, S, y, post, cm):
        """stream_i <- post_i * y + sum_j comb[j][i] * stream_j."""
        out = post.unsqueeze(-1) * y.unsqueeze(1) + torch.einsum("tji,tjd->tid", cm, S)
        return _bf(out) if self.emu else out

    def block_hc(self, pre, kind, is_moe, S, pos):
        x, post, cm = self.hc_pre(f"{pre}.hc_attn", S)
        h = self.norm(x, self.t[f"{pre}.attn_norm.weight"])
        if kind == "attention":
            a = self.attention(pre, h, pos)
        else:
            from .deltanet import reference_deltanet_layer
            a = reference_deltanet_layer(self, pre, h)
        S = self.hc_post(S, _bf(a) if self.emu else a, post, cm)
        x, post, cm = self.hc_pre(f"{pre}.hc_mlp", S)
        h = self.norm(x, self.t[f"{pre}.mlp_norm.weight"])
        m = self.moe(pre, h) if is_moe else self.swiglu(h, f"{pre}.mlp")
        return self.hc_post(S, _bf(m) if self.emu else m, post, cm)

    def block(self, pre, kind, is_moe, x, pos):
        h = self.norm(x, self.t[f"{pre}.attn_norm.weight"])
        if kind == "attention":
            a = self.attention(pre, h, pos)
        else:
            from .deltanet import reference_deltanet_layer
            a = reference_deltanet_layer(self, pre, h)
        x = x + a
        if self.emu:
            x = _bf(x)
        h = self.norm(x, self.t[f"{pre}.mlp_norm.weight"])
        if is_moe:
            m = self.moe(pre, h)
        else:
            m = self.swiglu(h, f"{pre}.mlp")
        x = x + m
        return _bf(x) if self.emu else x

    def hidden_prenorm(self, ids: torch.Tensor) -> torch.Tensor:
        """Last-layer hidden states [T, d] (before the final norm) of one sequence."""
        c = self.cfg
        x = self.t["embed.weight"].float()[ids]
        pos = torch.arange(ids.shape[0])
        if c.hc_streams:
            S = x.unsqueeze(1).expand(x.shape[0], c.hc_streams, x.shape[1]).clone()
            for i in range(c.num_layers):
                S = self.block_hc(f"layers.{i}", c.layer_kind(i), c.is_moe_layer(i), S, pos)
            x = S.mean(1)
            return _bf(x) if self.emu else x
        for i in range(c.num_layers):
            x = self.layer(i, x, pos)
        return x

    def hidden(self, ids: torch.Tensor) -> torch.Tensor:
        """Final-normed hidden states [T, d] of one sequence `ids` [T]."""
        return self.norm(self.hidden_prenorm(ids), self.t["final_norm.weight"])

    def head(self, h: torch.Tensor) -> torch.Tensor:
        w = self.W("lm_head")
        if self.emu and self.is_nv("lm_head"):
            return _qact(h) @ w.t()  # the GPU rounds the final-normed rows to NVFP4 for an NVFP4 head
        return (_bf(h) if self.emu else h) @ w.t()

    def logits(self, ids: torch.Tensor) -> torch.Tensor:
        return self.head(self.hidden(ids))

    def hidden_taps(self, ids: torch.Tensor) -> torch.Tensor:
        """The residual stream after every layer in cfg.mtp_taps, concatenated [T, n*d]."""
        c = self.cfg
        x = self.t["embed.weight"].float()[ids]
        pos = torch.arange(ids.shape[0])
        taps = {}
        for i in range(c.num_layers):
            x = self.layer(i, x, pos)
            taps[i] = x
        return torch.cat([taps[i] for i in c.mtp_taps], -1)

    def mtp(self, h: torch.Tensor, next_ids: torch.Tensor, j: int = 0, taps: torch.Tensor | None = None):
        """Multi-token-prediction head j over one sequence: row p pairs the target's
        pre-norm hidden state h[p] with the token at p+1 and predicts the token at
        p+2.  With mtp_taps, head 0 reads tap_proj(taps) (the concatenated tapped
        states) in place of h.  Returns (pre-norm MTP hidden [T, d], logits [T, V])."""
        pre = f"mtp.{j}"
        if taps is not None:
            h = self.lin(taps, f"{pre}.tap_proj")
            if self.emu:
                h = _bf(h)
        e = self.t["embed.weight"].float()[next_ids]
        en = self.norm(e, self.t[f"{pre}.enorm.weight"])
        hn = self.norm(h, self.t[f"{pre}.hnorm.weight"])
        x = self.lin(torch.cat([en, hn], -1), f"{pre}.eh_proj")
        if self.emu:
            x = _bf(x)
        pos = torch.arange(h.shape[0])
        x = self.block(f"{pre}.layer", "attention", self.cfg.num_experts > 0, x, pos)
        return x, self.head(self.norm(x, self.t[f"{pre}.norm.weight"]))

    @torch.no_grad()
    def generate(self, prompt: list[int], n: int) -> list[int]:
        ids = list(prompt)
        for _ in range(n):
            lg = self.logits(torch.tensor(ids))[-1]
            ids.append(int(lg.argmax()))
        return ids[len(prompt):]
