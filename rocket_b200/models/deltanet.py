"""Gated DeltaNet layers (Qwen3-Next hybrid): fuel tensors, CPU oracle, engine
weights and the GPU forward.

Layer (per token, v head h, qk head h // (Hv/Hk)):
    [q|k|v|z|b|a] = in_proj(x)
    q, k, v = silu(causal_conv4([q|k|v]))           (depthwise, over the sequence)
    q = l2norm(q) / sqrt(Dk);  k = l2norm(k)
    beta = sigmoid(b);  g = -exp(A_log) * softplus(a + dt_bias)
    S = exp(g) S;  S += beta k (v - S^T k)^T;  o = S^T q        (S: [Dk, Dv] fp32)
    y = out_proj( rmsnorm(o) * norm_w * silu(z) )

Kimi delta attention (KDA, ``deltanet.gate: channel``): the "a" block is f [Hv*Dk]
and the decay is per key channel, g[h, i] = lb * sigmoid(exp(A_log[h]) * (f[h, i] +
dt_bias[h, i])), S = diag(exp(g)) S; with ``out_gate: sigmoid`` the output gate is
sigmoid(z) (engines/glm5-moe-nvfp4-2b/src/kernels.cu:375-530: kda_forget,
kda_step, kda_gated_norm).

The recurrent state (and the last 3 conv inputs) of every running sequence
lives in a per-slot buffer; a sequence starting at position 0 starts from zero.

Reference counterparts: KDA layer run_kda (engines/glm5-moe-nvfp4-2b/src/
model.cu:1010) and the Qwen GDN core (engines/qwen38-flash-next-nvfp4-2b/src/
linear_attention/gdn_core.h:12-47).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .. import ops


def _dims(cfg, tp: int = 1):
    dn = cfg.deltanet
    Hk, Hv, D = dn.num_qk_heads // tp, dn.num_v_heads // tp, dn.head_dim
    return Hk, Hv, D, dn.conv_kernel


def _gw(cfg) -> int:
    """Width of one v head's gate input / log decay: 1 (per head) or Dk (per channel)."""
    return cfg.deltanet.head_dim if cfg.deltanet.gate == "channel" else 1


def init_deltanet_tensors(cfg, pre, t, m, g, lin, one):
    """Fuel-format DeltaNet tensors of layer `pre` (see weights.init_fuel_tensors)."""
    Hk, Hv, D, K = _dims(cfg)
    d = cfg.d_model
    lin(f"{pre}.dn.in_proj_qkvz", 2 * Hk * D + 2 * Hv * D, d, "attention")
    gw = _gw(cfg)
    lin(f"{pre}.dn.in_proj_ba", Hv + Hv * gw, d, "attention")   # b [Hv] | a [Hv] or f [Hv*Dk]
    C = 2 * Hk * D + Hv * D
    t[f"{pre}.dn.conv1d.weight"] = (torch.randn(C, K, generator=g) * (1.0 / math.sqrt(K))).bfloat16()
    t[f"{pre}.dn.A_log"] = torch.log(torch.empty(Hv).uniform_(1, 16, generator=g))
    t[f"{pre}.dn.dt_bias"] = torch.ones(Hv * gw)
    t[f"{pre}.dn.norm.weight"] = torch.ones(D).bfloat16()
    lin(f"{pre}.dn.out_proj", d, Hv * D, "attention")


def chunked_gated_delta_rule(q, k, v, g, beta, S0, chunk: int = 64):
    """The gated delta rule of one head in chunk form (the algebra a tensor-core prefill
    kernel evaluates), equal to the token-by-token recurrence up to rounding.

    q, k [T, Dk]; v [T, Dv]; g [T] (per-head log decay) or [T, Dk] (per-channel, KDA);
    beta [T]; S0 [Dk, Dv].  Returns (outputs [T, Dv], final state [Dk, Dv]).

    Per token: S_t = D_t S_{t-1} + k_t u_t^T with u_t = beta_t (v_t - (D_t S_{t-1})^T k_t),
    D_t = diag(exp(g_t)).  Inside a chunk with cumulative log decays G_t (G_0 = 0):
        A[t, i] = beta_t sum_c k_t[c] k_i[c] exp(G_t[c] - G_i[c])     (i < t)
        T = (I + A)^-1                           (unit lower triangular)
        U = T diag(beta) V - T diag(beta) K~ S0,  K~_t = exp(G_t) * k_t
        O = Q~ S0 + (tril(Q~ . K^ ) ) U,  Q~_t = exp(G_t) * q_t,  K^_i = exp(-G_i) * k_i
        S_C = exp(G_C) * S0 + sum_i exp(G_C - G_i) * k_i u_i^T
    Pairwise terms use exp(G_t - G_i) (<= 1 for i <= t) instead of the separate factors,
    so strong decays over a long chunk cannot overflow.
    """
    T, Dk = k.shape
    per_ch = g.dim() == 2
    S = S0.clone()
    outs = []
    for c0 in range(0, T, chunk):
        qc, kc, vc, bc = q[c0:c0 + chunk], k[c0:c0 + chunk], v[c0:c0 + chunk], beta[c0:c0 + chunk]
        gc = g[c0:c0 + chunk]
        n = qc.shape[0]
        G = torch.cumsum(gc, 0)                              # [n] or [n, Dk]
        low = torch.ones(n, n, dtype=torch.bool, device=q.device).tril()
        if per_ch:
            diff = G[:, None, :] - G[None, :, :]             # [t, i, c]
            dec = torch.where(low[:, :, None], torch.exp(torch.where(low[:, :, None], diff, torch.zeros_like(diff))),
                              torch.zeros_like(diff))
            kk = torch.einsum("tc,ic,tic->ti", kc, kc, dec)
            qk = torch.einsum("tc,ic,tic->ti", qc, kc, dec)
            kt = torch.exp(G) * kc
            qt = torch.exp(G) * qc
            tail = torch.exp(G[-1][None, :] - G) * kc          # exp(G_C - G_i) * k_i
            gC = torch.exp(G[-1])[:, None]                     # per key channel
        else:
            diff = G[:, None] - G[None, :]
            dec = torch.where(low, torch.exp(torch.where(low, diff, torch.zeros_like(diff))), torch.zeros_like(diff))
            kk = (kc @ kc.t()) * dec
            qk = (qc @ kc.t()) * dec
            kt = torch.exp(G)[:, None] * kc
            qt = torch.exp(G)[:, None] * qc
            tail = torch.exp(G[-1] - G)[:, None] * kc
            gC = torch.exp(G[-1])
        A = (bc[:, None] * kk).tril(-1)
        Tm = torch.linalg.solve_triangular(torch.eye(n, dtype=q.dtype, device=q.device) + A,
                                           torch.eye(n, dtype=q.dtype, device=q.device), upper=False,
                                           unitriangular=True)
        U = Tm @ (bc[:, None] * vc) - Tm @ (bc[:, None] * kt) @ S
        outs.append(qt @ S + qk @ U)
        S = gC * S + tail.t() @ U
    return torch.cat(outs), S


def reference_deltanet_layer(ref, lpre, x):
    """CPU fp32 oracle of one DeltaNet layer (tensors under `lpre`.dn) over a whole sequence x [T, d]."""
    c = ref.cfg
    Hk, Hv, D, K = _dims(c)
    T = x.shape[0]
    pre = f"{lpre}.dn"
    pz = ref.lin(x, f"{pre}.in_proj_qkvz")
    pba = ref.lin(x, f"{pre}.in_proj_ba")
    if ref.emu:
        pz, pba = pz.bfloat16().float(), pba.bfloat16().float()
    C = 2 * Hk * D + Hv * D
    conv_in = pz[:, :C]
    z = pz[:, C:C + Hv * D]
    w = ref.t[f"{pre}.conv1d.weight"].float()  # [C, K]
    xp = torch.cat([torch.zeros(K - 1, C), conv_in], 0)
    conv = torch.stack([(xp[s:s + K] * w.t()).sum(0) for s in range(T)])
    conv = F.silu(conv)
    q = conv[:, :Hk * D].view(T, Hk, D)
    k = conv[:, Hk * D:2 * Hk * D].view(T, Hk, D)
    v = conv[:, 2 * Hk * D:].view(T, Hv, D)
    q = q * torch.rsqrt((q * q).sum(-1, keepdim=True) + 1e-6) / math.sqrt(D)
    k = k * torch.rsqrt((k * k).sum(-1, keepdim=True) + 1e-6)
    beta = torch.sigmoid(pba[:, :Hv])
    A = torch.exp(ref.t[f"{pre}.A_log"].float())
    dtb = ref.t[f"{pre}.dt_bias"].float()
    if c.deltanet.gate == "channel":
        f = pba[:, Hv:Hv + Hv * D].view(T, Hv, D)
        gg = c.deltanet.gate_lower_bound * torch.sigmoid(A.view(1, Hv, 1) * (f + dtb.view(1, Hv, D)))
    else:
        gg = (-A * F.softplus(pba[:, Hv:2 * Hv] + dtb)).view(T, Hv, 1)
    rep = Hv // Hk
    S = torch.zeros(Hv, D, D)
    out = torch.zeros(T, Hv, D)
    for s in range(T):
        for h in range(Hv):
            kk, qq = k[s, h // rep], q[s, h // rep]
            S[h] = torch.exp(gg[s, h]).unsqueeze(1) * S[h]   # rows of S are key channels
            u = v[s, h] - S[h].t() @ kk
            S[h] = S[h] + beta[s, h] * torch.outer(kk, u)
            out[s, h] = S[h].t() @ qq
    nw = ref.t[f"{pre}.norm.weight"].float()  # the gated norm weight is plain (not zero-centred)
    zz = z.view(T, Hv, D)
    gate = torch.sigmoid(zz) if c.deltanet.out_gate == "sigmoid" else F.silu(zz)
    y = out * torch.rsqrt(out.pow(2).mean(-1, keepdim=True) + c.norm_eps) * nw * gate
    y = y.reshape(T, Hv * D)
    if ref.emu:
        y = y.bfloat16().float()
    return ref.lin(y, f"{pre}.out_proj")


@dataclass
class DeltaNetWeights:
    w_in: torch.Tensor      # [rows_pad, d] bf16: q|k|v|z|b|a (local heads)
    conv_w: torch.Tensor    # [C, K] bf16
    A_log: torch.Tensor     # [Hv] f32
    dt_bias: torch.Tensor   # [Hv] f32
    norm_w: torch.Tensor    # [D] bf16
    w_out: torch.Tensor     # [d, Hv*D] bf16
    index: int = 0          # DeltaNet layer ordinal (state buffer index)

    def nbytes(self):
        return sum(x.numel() * x.element_size() for x in (self.w_in, self.conv_w, self.A_log, self.dt_bias,
                                                          self.norm_w, self.w_out))


class DeltaNetBuffers:
    """Scratch and per-slot recurrent state of all DeltaNet layers of a model."""

    def __init__(self, cfg, par, max_tokens, max_slots, dev, spec_rows: int = 0):
        Hk, Hv, D, K = _dims(cfg, par.tp)
        self.Hk, self.Hv, self.D, self.K = Hk, Hv, D, K
        n = sum(1 for i in range(cfg.num_layers) if cfg.layer_kind(i) == "deltanet")
        self.n_layers = n
        C = 2 * Hk * D + Hv * D
        self.C = C
        self.gate_ch = cfg.deltanet.gate == "channel"
        gw = _gw(cfg)
        self.rows = C + Hv * D + Hv + Hv * gw
        self.rows_pad = (self.rows + 127) // 128 * 128
        f32 = dict(dtype=torch.float32, device=dev)
        self.proj = torch.zeros(max_tokens, self.rows_pad, dtype=torch.bfloat16, device=dev)
        self.q = torch.zeros(max_tokens, Hk, D, **f32)
        self.k = torch.zeros(max_tokens, Hk, D, **f32)
        self.v = torch.zeros(max_tokens, Hv, D, **f32)
        self.beta = torch.zeros(max_tokens, Hv, **f32)
        self.g = torch.zeros(max_tokens, Hv * gw, **f32)
        self.out = torch.zeros(max_tokens, Hv * D, dtype=torch.bfloat16, device=dev)
        self.o_raw = torch.zeros(max_tokens, Hv, D, **f32)  # scan outputs before the gated norm
        self.state = torch.zeros(n, max_slots, Hv, D, D, **f32)  # [.., Dv, Dk]: column j contiguous
        self.conv_state = torch.zeros(n, max_slots, K - 1, C, dtype=torch.bfloat16, device=dev)
        # speculative verify rows: per-layer inputs retained for the commit of the accepted tokens
        R = spec_rows
        self.spec_rows = R
        if R:
            self.rk = torch.zeros(n, R, Hk, D, **f32)
            self.rv = torch.zeros(n, R, Hv, D, **f32)
            self.rg = torch.zeros(n, R, Hv * gw, **f32)
            self.rb = torch.zeros(n, R, Hv, **f32)
            self.rx = torch.zeros(n, R, C, dtype=torch.bfloat16, device=dev)

    def state_bytes_per_slot(self) -> int:
        return self.n_layers * (self.Hv * self.D * self.D * 4 + (self.K - 1) * self.C * 2)


def _shard_rows(cfg, par):
    Hk, Hv, D, _ = _dims(cfg, par.tp)
    Hk_all, Hv_all = cfg.deltanet.num_qk_heads, cfg.deltanet.num_v_heads
    r = par.tp_rank
    q = (r * Hk * D, (r + 1) * Hk * D)
    k = (Hk_all * D + r * Hk * D, Hk_all * D + (r + 1) * Hk * D)
    v = (2 * Hk_all * D + r * Hv * D, 2 * Hk_all * D + (r + 1) * Hv * D)
    z = (2 * Hk_all * D + Hv_all * D + r * Hv * D, 2 * Hk_all * D + Hv_all * D + (r + 1) * Hv * D)
    b = (r * Hv, (r + 1) * Hv)
    gw = _gw(cfg)
    a = (Hv_all + r * Hv * gw, Hv_all + (r + 1) * Hv * gw)
    return q, k, v, z, b, a


def load_deltanet(cfg, t, pre, par, dev, index=0):
    from .weights import dequant
    q, k, v, z, b, a = _shard_rows(cfg, par)
    Hk, Hv, D, _ = _dims(cfg, par.tp)
    wz = dequant(t, f"{pre}.dn.in_proj_qkvz")
    wba = dequant(t, f"{pre}.dn.in_proj_ba")
    rows = torch.cat([wz[q[0]:q[1]], wz[k[0]:k[1]], wz[v[0]:v[1]], wz[z[0]:z[1]], wba[b[0]:b[1]],
                      wba[a[0]:a[1]]]).bfloat16()
    n = rows.shape[0]
    w_in = torch.zeros((n + 127) // 128 * 128, rows.shape[1], dtype=torch.bfloat16)
    w_in[:n] = rows
    cw = t[f"{pre}.dn.conv1d.weight"]
    conv = torch.cat([cw[q[0]:q[1]], cw[k[0]:k[1]], cw[v[0]:v[1]]])
    wo = dequant(t, f"{pre}.dn.out_proj")[:, par.tp_rank * Hv * D:(par.tp_rank + 1) * Hv * D].bfloat16()
    gw = _gw(cfg)
    return DeltaNetWeights(w_in.to(dev), conv.contiguous().to(dev),
                           t[f"{pre}.dn.A_log"].float()[b[0]:b[1]].contiguous().to(dev),
                           t[f"{pre}.dn.dt_bias"].float()[b[0] * gw:b[1] * gw].contiguous().to(dev),
                           t[f"{pre}.dn.norm.weight"].to(dev), wo.contiguous().to(dev), index)


def random_deltanet(cfg, par, gen, dev, index=0):
    Hk, Hv, D, K = _dims(cfg, par.tp)
    d = cfg.d_model
    std = cfg.init_std
    C = 2 * Hk * D + Hv * D
    gw = _gw(cfg)
    rows = C + Hv * D + Hv + Hv * gw
    bf = dict(dtype=torch.bfloat16, device=dev)
    w_in = torch.zeros((rows + 127) // 128 * 128, d, **bf)
    w_in[:rows] = torch.randn(rows, d, generator=gen, **bf) * std
    conv = torch.randn(C, K, generator=gen, **bf) / math.sqrt(K)
    A_log = torch.log(torch.rand(Hv, generator=gen, device=dev) * 15 + 1)
    dt_bias = torch.ones(Hv * gw, device=dev)
    return DeltaNetWeights(w_in, conv, A_log, dt_bias, torch.ones(D, **bf),
                           torch.randn(d, Hv * D, generator=gen, **bf) * std, index)


def deltanet_forward(model, i, L, xn, x, T, S, decode, lead, meta, spec_rows: int = 0):
    buf = model.dn_buf
    w = L.dn
    c = model.cfg
    ops.linear_bf16(xn, w.w_in, out=buf.proj[:T])
    li = w.index
    if spec_rows > buf.spec_rows:
        raise ValueError(f"{spec_rows} verify rows > the {buf.spec_rows} retained rows")
    r = (buf.rk[li], buf.rv[li], buf.rg[li], buf.rb[li], buf.rx[li]) if spec_rows else (None,) * 5
    ops.ext().gdn(buf.proj[:T], w.conv_w, buf.conv_state[li], w.A_log, w.dt_bias, w.norm_w, buf.q, buf.k, buf.v,
                  buf.beta, buf.g, buf.state[li], buf.out, meta.pos, meta.q_start, meta.q_len, meta.state_slot,
                  buf.Hk, buf.Hv, buf.K, buf.C, float(c.norm_eps), T, S, spec_rows, *r,
                  int(buf.gate_ch), float(c.deltanet.gate_lower_bound), int(c.deltanet.out_gate == "sigmoid"),
                  buf.o_raw, 1)
    if lead:
        ops.linear_bf16(buf.out[:T], w.w_out, out=x, epi=ops.EPI_RESIDUAL_BF16, residual=x)
    else:
        ops.linear_bf16(buf.out[:T], w.w_out, out=x)
