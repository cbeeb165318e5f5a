"""Replicated-token multi-GPU step with every collective fused into the kernels around it.

Every rank holds the residual rows of all T tokens of the step.  Attention heads, the
dense-MLP intermediate and the vocabulary are tensor parallel (TP = N, or replicated
with TP = 1); routed experts are expert parallel (EP = N).  Per layer:

  land(previous push) + RMSNorm         fixed-order sum of the pushed rows + residual
  QKV GEMM -> RoPE + paged KV write -> decode attention (this rank's heads)
  o_proj GEMM, epilogue pushes bf16 partial rows to every rank    (GEMM -> all-reduce)
  land(all-reduce) + RMSNorm
  router GEMM + top-k (all tokens, this rank's experts) -> plan -> dispatch quantize
  grouped GEMM1 (SwiGLU) -> NVFP4 -> grouped GEMM2, then
    TP = 1: its epilogue pushes every expert output row (token, routing slot) into that
            slot of every rank's combine buffer                    (GEMM -> combine)
            (the next layer's land sums the slots with moe_combine_kernel's fma chain)
    TP > 1: one combine kernel sums this rank's slots and pushes one partial row per
            token (an all-reduce, landed like the o_proj one)

Two syncs per layer; every rank lands the same bits, so the replicated residual never
diverges.  With TP = 1 (attention replicated) there is no all-reduce and the step
reproduces the single-GPU step bit for bit: the exact-parity layout of `static-fire`.

The shared expert of layer i is computed by rank i mod N (its weights are on every
rank), spreading its bytes over the ranks.

Buffers: three rotating buffers in a symmetric heap, each [max(N, k_out)][T][d] bf16.
A rank may push sync s+1 while a slower rank still lands sync s (it has passed s's
wait, not the peer's read), never sync s-1; so consecutive syncs use different
buffers.  The first sync of every step uses buffer 2 and the rest alternate 0 / 1, so a
step's first push never lands on the buffer the previous step's last sync used.

Only the vocab-parallel argmax keys use NCCL (one small MAX all-reduce per step under
TP > 1).  Peer memory is touched only by plain stores in the GEMM epilogues; TMA
tensor maps stay local and no load of this path is a multicast.

Reference counterparts: the expert-parallel row exchange
(engines/glm5-moe-nvfp4-2b/src/fabric/expert_parallel.h:51-130) with its host sync per
MoE layer (src/model.cu:1976-1980), and the static-fire parity gate that requires zero
mismatched tokens between one and two ranks (src/fabric/static_fire.cu:1-18).
"""
from __future__ import annotations

import torch

from .. import ops
from ..parallel.symm import SymmetricHeap

SITE = 0          # one epoch site: producer and consumer launches strictly alternate
HEAP_SLOT = 1     # peer-pointer registry slot (the sequence-parallel path uses 0)
LAND_NONE, LAND_COMB, LAND_AR = 0, 2, 3


class ArFused:
    def __init__(self, model, max_tokens: int):
        m = model
        c = m.cfg
        par = m.par
        self.m = m
        self.N, self.rank = par.world, par.rank
        self.tp = par.tp
        self.Tm = max_tokens
        d = c.d_model
        self.d = d
        self.k_out = (c.top_k + c.num_shared_experts) if c.num_experts else 1
        self.slots = max(self.N, self.k_out)
        elems = self.slots * self.Tm * d
        self.heap = SymmetricHeap(par, 3 * (elems * 2 + 1024), slot=HEAP_SLOT)
        self.off = [self.heap.alloc(elems * 2) for _ in range(3)]
        self.buf = [self.heap.view(o, (elems,), torch.bfloat16) for o in self.off]
        dev = m.dev
        if c.num_experts:
            rows = max(m.plan_dec.max_rows, m.plan_pre.max_rows)
            self.row_meta = torch.full((rows,), -1, dtype=torch.int32, device=dev)
            # the plan choice follows the single-GPU rule (all experts), so a replicated-attention
            # step tiles every expert GEMM exactly as one GPU does
            self.e_all = c.num_experts + c.num_shared_experts
        self.err = ops.err_flag(dev)
        self._k = 0       # sync index within the current step
        self.pending = None

    def handles(self, T: int, n_out: int) -> bool:
        return T <= self.Tm

    # ------------------------------------------------------------------ syncs
    def _next_buf(self) -> int:
        b = 2 if self._k == 0 else (self._k - 1) % 2
        self._k += 1
        return b

    def _land(self, T: int, norm_w):
        """x[:T] (+)= the pending push (if any); xn[:T] = RMSNorm(x) when norm_w is given."""
        m, c = self.m, self.m.cfg
        p = self.pending
        self.pending = None
        x = m.x[:T]
        xn = m.xn if norm_w is not None else None
        if p is None:
            if norm_w is not None:
                ops.rmsnorm(x, norm_w, c.norm_eps, c.zero_centered_norm, out=m.xn[:T])
            return
        mode, b, comb_w = p
        buf = self.buf[b]
        ops.ext().ar_land(m.x, T, mode, norm_w, xn, c.norm_eps, c.zero_centered_norm,
                          buf if mode == LAND_AR else None, self.Tm, self.N,
                          buf if mode == LAND_COMB else None, comb_w, self.k_out, SITE, HEAP_SLOT, self.err)

    def _push_args(self, epi: int, b: int, **kw) -> dict:
        f = {"peer_slot": HEAP_SLOT, "signal_site": SITE}
        if epi == ops.EPI_AR_PUSH:
            f.update(ar_off=self.off[b], ar_rows=self.Tm)
        else:
            f.update(comb_off=self.off[b], k_out=self.k_out, meta=self.row_meta.data_ptr())
        f.update(kw)
        return f

    def _linear_push(self, x, w, T, xq):
        """Partial rows of x @ w^T pushed to slot `rank` of every rank's all-reduce buffer."""
        b = self._next_buf()
        f = self._push_args(ops.EPI_AR_PUSH, b)
        out = self.buf[b]  # not written locally by this epilogue; any bf16 tensor will do
        # split K like the plain GEMM would (a decode-sized projection fills few SMs
        # otherwise); the split reduce then pushes the summed rows and signals
        if isinstance(w, ops.Fp8Weight):
            ops.quantize_rows_fp8(x, xq, T)
            s = ops.pick_splits(T, w.n, w.k // 2, False)
            ops.linear_fp8(xq, T, w, out=out, epi=ops.EPI_AR_PUSH, splits=s, fused=f)
        elif isinstance(w, ops.NvFp4Weight):
            ops.quantize_rows(x, xq, T)
            s = ops.pick_splits(T, w.n, w.k, True)
            ops.linear_nvfp4(xq, T, w, out=out, epi=ops.EPI_AR_PUSH, splits=s, fused=f)
        else:
            s = ops.pick_splits(T, w.shape[0], w.shape[1], False)
            ops.linear_bf16(x, w, out=out, epi=ops.EPI_AR_PUSH, splits=s, fused=f)
        self.pending = (LAND_AR, b, None)

    # ------------------------------------------------------------------ step
    def forward(self, T: int, S: int, W_: int, n_out: int, decode: bool, logits_out=None) -> torch.Tensor:
        m, c = self.m, self.m.cfg
        meta = m.main_meta()
        x = m.x[:T]
        tm = m.timer
        self._k = 0
        self.pending = None
        tm.start("embed")
        ops.embed(meta.ids[:T], m.embed, x, 0)
        tm.stop("embed")
        for i, L in enumerate(m.layers):
            m._cur_layer = i
            m._n_seqs = S
            tm.start("land+norm")
            self._land(T, L.attn_norm)
            tm.stop("land+norm")
            if i:
                m.capture_tap(i - 1, x, T)  # x now holds layer i-1's output
            self._attention(i, L, T, W_, decode, meta)
            tm.start("land+norm")
            self._land(T, L.mlp_norm)
            tm.stop("land+norm")
            if L.moe:
                self._moe(i, L, T, decode)
            else:
                tm.start("dense_mlp")
                self._dense(L, T)
                tm.stop("dense_mlp")
            if m.telemetry is not None:
                self._land(T, None)
                m.telemetry.layer(i, x)
        tm.start("land+norm")
        self._land(T, None)
        tm.stop("land+norm")
        m.capture_tap(len(m.layers) - 1, x, T)
        tm.start("lm_head")
        xs = torch.index_select(x, 0, m.out_rows[:n_out], out=m.x_last[:n_out])
        out = m._head(xs, n_out, m.final_norm, m.out_ids[:n_out], logits_out)
        tm.stop("lm_head")
        return out

    def _attention(self, i, L, T, W_, decode, meta):
        m, c, tm = self.m, self.m.cfg, self.m.timer
        D = c.head_dim
        xn = m.xn[:T]
        tm.start("attn.qkv")
        qkv = m._linear(xn, L.wqkv, m.qkv[:T], T=T, xq=m.xq_attn)
        if L.qkv_bias is not None:
            qkv[:, :L.qkv_bias.numel()].add_(L.qkv_bias)
        tm.stop("attn.qkv")
        li = m.attn_index[i]
        tm.start("attn.rope_kv")
        ops.qk_rope_kv(qkv, T, m.Hq, m.Hkv, D, c.rotary_dim, c.attn_output_gate, meta.pos[:T], m.inv_freq,
                       m.q[:T], m.gate[:T] if m.gate is not None else None, L.q_norm, L.k_norm, c.norm_eps,
                       c.zero_centered_norm, m.k_cache[li], m.v_cache[li], meta.slots[:T], m.page_size,
                       m.k_scales[li], m.v_scales[li])
        tm.stop("attn.rope_kv")
        m._dense_attention(li, T, W_, decode, meta)
        tm.start("attn.o")
        if self.tp > 1:
            self._linear_push(m.attn_out[:T], L.wo, T, m.xq_attn_o)
        else:
            x = m.x[:T]
            m._linear(m.attn_out[:T], L.wo, x, epi=ops.EPI_RESIDUAL_BF16, residual=x, T=T, xq=m.xq_attn_o)
        tm.stop("attn.o")

    def _dense(self, L, T):
        m = self.m
        xn, x = m.xn[:T], m.x[:T]
        if self.tp == 1:
            m._dense(L, xn, x, T, True)
            return
        ops.quantize_rows(xn, m.xq_d, T)
        ops.linear_nvfp4(m.xq_d, T, L.w13, out=m.hd[:T], epi=ops.EPI_SWIGLU)
        self._linear_push(m.hd[:T], L.w2, T, m.hq_d)

    def _moe(self, i, L, T, decode):
        m, c, tm = self.m, self.m.cfg, self.m.timer
        xn = m.xn[:T]
        few = T * self.k_out <= 32 * self.e_all
        plan = m.plan_dec if (T <= m.plan_dec_tokens and (decode or few)) else m.plan_pre
        tm.start("moe.router")
        logits = ops.linear_bf16(xn, L.router_w, out=m.logits[:T], epi=ops.EPI_STORE_F32)
        ops.route_and_plan(logits, c.num_experts, c.top_k, c.num_shared_experts, c.router == "sigmoid",
                           c.norm_topk_prob, c.routed_scaling, L.router_b,
                           c.num_experts if c.shared_expert_gate else -1, plan, T,
                           e_lo=m.e_lo, e_hi=m.e_lo + m.E_l, shared_local=(i % self.N) == self.rank)
        tm.stop("moe.router")
        exact = self.tp == 1
        tm.start("moe.dispatch")
        ops.moe_dispatch_quantize(xn, T, plan, m.xq, row_meta=self.row_meta if exact else None)
        tm.stop("moe.dispatch")
        tm.start("moe.gemm1")
        ops.grouped_nvfp4(m.xq, L.w13, m.h, ops.EPI_SWIGLU, plan, plan.bn)
        tm.stop("moe.gemm1")
        tm.start("moe.quant_h")
        ops.quantize_assigned(m.h, T, plan, m.hq)
        tm.stop("moe.quant_h")
        b = self._next_buf()
        if exact:
            # every expert row goes to every rank: the land sums all routing slots in the
            # single-GPU order, so the step reproduces one GPU bit for bit
            tm.start("moe.gemm2(comb push)")
            ops.grouped_nvfp4(m.hq, L.w2, self.buf[b], ops.EPI_COMBINE_ALL, plan, plan.bn,
                              fused=self._push_args(ops.EPI_COMBINE_ALL, b))
            tm.stop("moe.gemm2(comb push)")
            self.pending = (LAND_COMB, b, plan.weights)
        else:
            # tensor-parallel layout: this rank's slots summed locally, one partial row per
            # token pushed (an all-reduce; a ninth of the NVLink bytes of the row push)
            tm.start("moe.gemm2")
            ops.grouped_nvfp4(m.hq, L.w2, m.y, ops.EPI_STORE_BF16, plan, plan.bn)
            tm.stop("moe.gemm2")
            tm.start("moe.combine(push)")
            ops.ext().moe_combine_push(m.y, plan.pos, plan.weights, self.k_out, T, self.off[b], self.Tm, HEAP_SLOT,
                                       SITE)
            tm.stop("moe.combine(push)")
            self.pending = (LAND_AR, b, None)
