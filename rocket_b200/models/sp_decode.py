"""Sequence-parallel decode step with collectives fused into the compute kernels.

Layout: a decode batch of B tokens (B divisible by the world size N) is split
so rank r owns the residual rows of tokens [r*T_r, (r+1)*T_r), T_r = B/N.
Attention heads, the dense-MLP intermediate and the vocabulary are tensor
parallel; routed experts are expert parallel.  Per layer:

  land(..) -> RMSNorm -> push xn rows to every rank         (norm + all-gather)
  QKV GEMM, TMA producer waits for the gathered rows         (all-gather -> GEMM)
  RoPE + paged KV write, decode attention (local heads, all B sequences)
  o_proj GEMM, epilogue pushes fp32 partial rows to owners   (GEMM -> reduce-scatter)
  land(RS) -> residual + RMSNorm (local)                     (reduce-scatter landing)
  MoE: router GEMM on T_r rows -> dispatch kernel: top-k, NVFP4 quantize, push
       each routed row into its expert owner's slot          (dispatch all-to-all)
       owner: plan -> grouped GEMM1 (SwiGLU) -> NVFP4 -> grouped GEMM2 whose
       epilogue pushes every output row back to its source (combine all-to-all)
  land(COMB) -> weighted sum (fixed slot order) + residual + next RMSNorm + push
  dense layers: land(RS) -> NVFP4 all-gather -> w13 GEMM (waits) -> w2 GEMM (RS push)

Only the vocab-parallel argmax keys use NCCL (one small MAX all-reduce per
step).  Every wait is bounded (comm.cuh); nothing here uses TMA multicast or
hands peer memory to a library kernel.
"""
from __future__ import annotations

import torch

from .. import ops
from ..parallel.symm import SymmetricHeap

AG, RS, DISP, COMB = 0, 1, 2, 3
LAND_NONE, LAND_RS, LAND_COMB = 0, 1, 2
OUT_LOCAL, OUT_AG, OUT_AG_NV = 0, 1, 2


class _HeapAct:
    """NvFp4Act-compatible views into the symmetric heap."""

    def __init__(self, packed, sf, row_scale, k):
        self.packed, self.sf, self.row_scale, self.k = packed, sf, row_scale, k
        self.rows = packed.shape[0]


class SpDecode:
    def __init__(self, model, max_batch: int, rs_splits: int = 4):
        m = model
        c = m.cfg
        self.m = m
        par = m.par
        self.N = par.world
        self.rank = par.rank
        self.max_batch = (max_batch + self.N - 1) // self.N * self.N
        self.tr_max = self.max_batch // self.N
        self.rs_splits = rs_splits
        self.rs_n = 1  # split count of the reduce-scatter partials currently in flight
        d = c.d_model
        self.d = d
        dev = m.dev
        self.k_out = c.top_k + c.num_shared_experts
        self.E_l = c.num_experts // self.N
        self.n_exp_local = self.E_l + c.num_shared_experts
        span = self.N * self.tr_max
        self.seg_rows = (span + 127) // 128 * 128
        self.moe_rows = self.n_exp_local * self.seg_rows
        I_l = c.dense_intermediate // m.par.tp if c.num_dense_layers else 0
        # ---- symmetric heap layout (identical on every rank)
        T = self.max_batch
        sizes = {}
        sizes["ag"] = T * d * 2
        sizes["agq"] = T * d // 2
        sizes["agsf"] = ((T + 127) // 128) * (d // 64) * 512
        sizes["agrs"] = T * 4
        sizes["rs"] = self.N * rs_splits * self.tr_max * d * 4
        sizes["xq"] = self.moe_rows * d // 2
        sizes["xsf"] = self.moe_rows // 128 * (d // 64) * 512
        sizes["xrs"] = self.moe_rows * 4
        sizes["meta"] = self.moe_rows * 4
        sizes["cnt"] = self.n_exp_local * 8 * 4
        sizes["comb"] = self.tr_max * self.k_out * d * 2
        total = sum(s + 1024 for s in sizes.values())
        self.heap = SymmetricHeap(par, total, slot=0)
        self.off = {k: self.heap.alloc(v) for k, v in sizes.items()}
        H = self.heap
        self.ag = H.view(self.off["ag"], (T, d), torch.bfloat16)
        self.agq = _HeapAct(H.view(self.off["agq"], (T, d // 2), torch.uint8),
                            H.view(self.off["agsf"], (sizes["agsf"],), torch.uint8),
                            H.view(self.off["agrs"], (T,), torch.float32), d)
        self.rs = H.view(self.off["rs"], (self.N * rs_splits, self.tr_max, d), torch.float32)
        self.xq = _HeapAct(H.view(self.off["xq"], (self.moe_rows, d // 2), torch.uint8),
                           H.view(self.off["xsf"], (sizes["xsf"],), torch.uint8),
                           H.view(self.off["xrs"], (self.moe_rows,), torch.float32), d)
        self.meta = H.view(self.off["meta"], (self.moe_rows,), torch.int32)
        self.cnt = H.view(self.off["cnt"], (self.n_exp_local, 8), torch.int32)
        self.comb = H.view(self.off["comb"], (self.tr_max, self.k_out, d), torch.bfloat16)
        # ---- local buffers
        bf = dict(dtype=torch.bfloat16, device=dev)
        i32 = dict(dtype=torch.int32, device=dev)
        self.x = torch.zeros(self.tr_max, d, **bf)
        self.xn = torch.zeros(self.tr_max, d, **bf)
        self.logits = torch.zeros(self.tr_max, m.E_pad if c.num_experts else 128, dtype=torch.float32, device=dev)
        self.comb_w = torch.zeros(self.tr_max, self.k_out, dtype=torch.float32, device=dev)
        self.cnt_local = torch.zeros(max(c.num_experts, 1), **i32)
        self.max_blocks = self.n_exp_local * ((span + 127) // 128)
        self.blk_expert = torch.zeros(self.max_blocks, **i32)
        self.blk_row = torch.zeros(self.max_blocks, **i32)
        self.blk_valid = torch.zeros(self.max_blocks, **i32)
        self.num_blocks = torch.zeros(1, **i32)
        self.row_list = torch.zeros(self.moe_rows, **i32)
        self.num_rows = torch.zeros(1, **i32)
        self.h = torch.zeros(self.moe_rows, c.moe_intermediate if c.num_experts else 64, **bf)
        self.hq = ops.NvFp4Act(self.moe_rows, c.moe_intermediate if c.num_experts else 64, dev)
        if I_l:
            self.hd = torch.zeros(T, I_l, **bf)
            self.hqd = ops.NvFp4Act(T, I_l, dev)
        self.err = ops.err_flag(dev)

    def handles(self, T: int, n_out: int) -> bool:
        return T % self.N == 0 and T <= self.max_batch and n_out == T

    # ------------------------------------------------------------------ pieces
    def _land(self, tr, mode, out, norm_w, wait=-1, signal=-1):
        c = self.m.cfg
        ops.ext().sp_land(self.x[:tr], norm_w, c.norm_eps, c.zero_centered_norm, tr, mode, out,
                          self.rs if mode == LAND_RS else None, self.N * self.rs_n,
                          self.comb if mode == LAND_COMB else None, self.comb_w if mode == LAND_COMB else None,
                          self.k_out, self.xn if out == OUT_LOCAL else None, self.off["ag"], self.off["agq"],
                          self.off["agsf"], self.off["agrs"], wait, signal, self.heap.slot, self.err)

    def _gemm(self, w, x_packed_or_bf16, out, epi, m_tokens, bn, xact=None, fused=None, grouped=None, splits=1):
        if isinstance(w, ops.NvFp4Weight):
            a = xact
            blk = grouped
            ops.ext().gemm(w.packed, a.packed, out, epi, w.n, w.k, m_tokens, bn, w.sf, a.sf, w.gscale, a.row_scale,
                           None, None, blk[0] if blk else None, blk[1] if blk else None, blk[2] if blk else None,
                           blk[3] if blk else None, blk[4] if blk else 0, w.num_experts, 1 << 30, self.err, 0,
                           splits, None, fused)
        else:
            ws = None
            if splits > 1 and epi not in (ops.EPI_REDUCE_SCATTER, ops.EPI_COMBINE_PUSH):
                ws = ops.splitk_workspace(self.m.dev, splits, m_tokens, w.shape[0])
            ops.ext().gemm(w, x_packed_or_bf16, out, epi, w.shape[0], w.shape[1], m_tokens, bn, None, None, None,
                           None, None, None, None, None, None, None, 0, 1, 1 << 30, self.err, 0, splits, ws, fused)

    def _rs_splits(self, n, k, nvf4):
        kt = k // (256 if nvf4 else 64)
        best = 1
        for s in range(1, self.rs_splits + 1):
            if kt // s >= 4 and (n // 128) * s <= ops.num_sms():
                best = s
        return best

    # ------------------------------------------------------------------ step
    def forward(self, B: int, W_: int, logits_out=None) -> torch.Tensor:
        m, c = self.m, self.m.cfg
        N, r = self.N, self.rank
        tr = B // N
        D = c.head_dim
        d = self.d
        slot = self.heap.slot
        tm = m.timer
        tm.start("sp.embed_land")
        ops.embed(m.ids[r * tr:(r + 1) * tr], m.embed, self.x[:tr], 0)
        self._land(tr, LAND_NONE, OUT_AG, m.layers[0].attn_norm, signal=AG)
        tm.stop("sp.embed_land")
        nl = len(m.layers)
        for i, L in enumerate(m.layers):
            nxt_norm = m.layers[i + 1].attn_norm if i + 1 < nl else m.final_norm
            # ---------------- attention (TP heads over all B tokens)
            tm.start("sp.qkv(wait AG)")
            self._gemm(L.wqkv, self.ag[:B], m.qkv[:B], ops.EPI_STORE_BF16, B, ops._bn_for(B),
                       splits=ops.pick_splits(B, L.wqkv.shape[0], d, False),
                       fused={"peer_slot": slot, "wait_site": AG})
            tm.stop("sp.qkv(wait AG)")
            tm.start("sp.rope_attn")
            li = m.attn_index[i]
            ops.qk_rope_kv(m.qkv[:B], B, m.Hq, m.Hkv, D, c.rotary_dim, c.attn_output_gate, m.pos[:B], m.inv_freq,
                           m.q[:B], m.gate[:B] if m.gate is not None else None, L.q_norm, L.k_norm, c.norm_eps,
                           c.zero_centered_norm, m.k_cache[li], m.v_cache[li], m.slots[:B], m.page_size,
                           m.k_scales[li], m.v_scales[li])
            ops.attention(m.q[:B], m.attn_out[:B].view(B, m.Hq, D), m.k_cache[li], m.v_cache[li], m.Hq, m.Hkv, D,
                          m.block_table, m.q_start, m.q_len, m.kv_len, m.w_seq, m.w_tok0, m.num_work, W_,
                          gate=m.gate[:B] if m.gate is not None else None, num_splits=m.splits,
                          ws_o=m.ws_o if m.splits > 1 else None, ws_ml=m.ws_ml if m.splits > 1 else None,
                          page_size=m.page_size, decode=True, k_scale=m.k_scales[li], v_scale=m.v_scales[li])
            tm.stop("sp.rope_attn")
            s = self._rs_splits(d, m.Hq * D, False)
            self.rs_n = s
            tm.start("sp.o_proj(RS push)")
            self._gemm(L.wo, m.attn_out[:B], self.rs, ops.EPI_REDUCE_SCATTER, B, ops._bn_for(B), splits=s,
                       fused={"peer_slot": slot, "signal_site": RS, "rs_off": self.off["rs"], "t_r": tr})
            tm.stop("sp.o_proj(RS push)")
            if L.moe:
                tm.start("sp.land_rs")
                self._land(tr, LAND_RS, OUT_LOCAL, L.mlp_norm, wait=RS)
                tm.stop("sp.land_rs")
                self._moe(L, tr, nxt_norm)
            else:
                tm.start("sp.dense")
                self._land(tr, LAND_RS, OUT_AG_NV, L.mlp_norm, wait=RS, signal=AG)
                self._gemm(L.w13, None, self.hd[:B], ops.EPI_SWIGLU, B, ops._bn_for(B), xact=self.agq,
                           fused={"peer_slot": slot, "wait_site": AG})
                ops.quantize_rows(self.hd[:B], self.hqd, B)
                s2 = self._rs_splits(d, L.w2.k, True)
                self.rs_n = s2
                self._gemm(L.w2, None, self.rs, ops.EPI_REDUCE_SCATTER, B, ops._bn_for(B), xact=self.hqd, splits=s2,
                           fused={"peer_slot": slot, "signal_site": RS, "rs_off": self.off["rs"], "t_r": tr})
                self._land(tr, LAND_RS, OUT_AG, nxt_norm, wait=RS, signal=AG)
                tm.stop("sp.dense")
        tm.start("sp.lm_head")
        # ---------------- vocab-parallel lm_head over the gathered final hidden states
        if logits_out is not None:  # numerics/debug: fp32 logits of this rank's vocab shard
            self._gemm(m.lm_head, self.ag[:B], logits_out[:B], ops.EPI_STORE_F32, B, ops._bn_for(B),
                       fused={"peer_slot": slot, "wait_site": AG})
            return logits_out[:B]
        keys = m.keys[:B]
        n_valid = min(m.V_l, c.vocab_size - m.v_lo)
        ops.ext().gemm(m.lm_head, self.ag[:B], keys, ops.EPI_ARGMAX, m.lm_head.shape[0], d, B, ops._bn_for(B), None,
                       None, None, None, None, None, None, None, None, None, 0, 1, n_valid, self.err, m.v_lo, 1, None,
                       {"peer_slot": slot, "wait_site": AG})
        if N > 1:
            keys.bitwise_xor_(-(1 << 63))
            m.par.all_reduce_max(keys)
            keys.bitwise_xor_(-(1 << 63))
        ops.argmax_finalize(keys, m.out_ids[:B])
        tm.stop("sp.lm_head")
        return m.out_ids[:B]

    def _moe(self, L, tr, nxt_norm):
        m, c = self.m, self.m.cfg
        slot = self.heap.slot
        d = self.d
        tm = m.timer
        tm.start("moe.router")
        ops.linear_bf16(self.xn[:tr], L.router_w, out=self.logits[:tr], epi=ops.EPI_STORE_F32)
        tm.stop("moe.router")
        args = {
            "logits": self.logits, "ld_logits": self.logits.shape[1], "E": c.num_experts, "top_k": c.top_k,
            "n_shared": c.num_shared_experts, "sigmoid": int(c.router == "sigmoid"), "norm_topk": int(c.norm_topk_prob),
            "shared_gate_col": c.num_experts if c.shared_expert_gate else -1, "scaling": float(c.routed_scaling),
            "bias": L.router_b, "xn": self.xn, "k": d, "comb_w": self.comb_w, "cnt_local": self.cnt_local,
            "seg_rows": self.seg_rows, "cap": self.tr_max, "xq_off": self.off["xq"], "sf_off": self.off["xsf"],
            "rs_off": self.off["xrs"], "meta_off": self.off["meta"], "cnt_off": self.off["cnt"],
            "signal_site": DISP, "blk_expert": self.blk_expert, "blk_row": self.blk_row, "blk_valid": self.blk_valid,
            "num_blocks": self.num_blocks, "row_list": self.row_list, "num_rows": self.num_rows, "err": self.err,
        }
        tm.start("moe.dispatch(push)")
        ops.ext().moe_dispatch_sp(args, slot, tr)
        tm.stop("moe.dispatch(push)")
        tm.start("moe.plan(wait DISP)")
        ops.ext().moe_owner_plan_sp(args, slot)
        tm.stop("moe.plan(wait DISP)")
        blk = (self.blk_expert, self.blk_row, self.blk_valid, self.num_blocks, self.max_blocks)
        tm.start("moe.gemm1")
        self._gemm(L.w13, None, self.h, ops.EPI_SWIGLU, 0, 128, xact=self.xq, grouped=blk)
        tm.stop("moe.gemm1")
        tm.start("moe.quant_h")
        ops.ext().quantize_rows_list(self.h, self.row_list, self.num_rows, self.hq.packed, self.hq.sf,
                                     self.hq.row_scale, 128, self.moe_rows)
        tm.stop("moe.quant_h")
        tm.start("moe.gemm2(comb push)")
        self._gemm(L.w2, None, self.h, ops.EPI_COMBINE_PUSH, 0, 128, xact=self.hq, grouped=blk,
                   fused={"peer_slot": slot, "signal_site": COMB, "comb_off": self.off["comb"], "k_out": self.k_out,
                          "seg_rows": self.seg_rows, "cap": self.tr_max, "counts": self.cnt,
                          "meta": self.meta.data_ptr()})
        tm.stop("moe.gemm2(comb push)")
        tm.start("moe.land_comb(AG push)")
        self._land(tr, LAND_COMB, OUT_AG, nxt_norm, wait=COMB, signal=AG)
        tm.stop("moe.land_comb(AG push)")
