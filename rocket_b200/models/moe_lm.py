"""GPU executor of the MoE decoder family (GLM-style GQA MoE, tiny oracle model,
Qwen3-Next hybrid via gated DeltaNet layers).

Every op is one of the framework's sm_100a kernels (``rocket_b200.ops``):

    embed -> per layer:
        rmsnorm -> QKV GEMM (bf16 or NVFP4) -> q/k norm + RoPE + paged KV write
        -> paged flash attention (tcgen05) -> O GEMM (+residual epilogue)
        rmsnorm -> router GEMM (fp32 out) -> top-k -> plan -> NVFP4 dispatch
        -> grouped GEMM1 (SwiGLU epilogue) -> NVFP4 -> grouped GEMM2 -> combine(+residual)
    -> final rmsnorm of the sampled rows -> lm_head GEMM with fused argmax

All activations live in static buffers sized for ``max_tokens`` so a decode
step can be captured once per batch bucket in a CUDA graph and replayed.

Parallelism (one process per GPU): attention heads, dense-MLP intermediate and
the vocabulary are sharded tensor-parallel; routed experts are sharded
expert-parallel with replicated routing.  Partial sums meet in an all-reduce
(the unfused path; see parallel/fused.py for the fused collectives).

Reference counterparts: DecodeEngine::step / run_mla / run_moe
(engines/glm5-moe-nvfp4-2b/src/model.cu:2331, 1381, 1876) and the Qwen TP2
layer adapters (engines/qwen38-flash-next-nvfp4-2b/src/decode/*.h).
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass

import torch

from .. import ops
from ..config import ModelConfig
from ..parallel.context import ParallelCtx
from ..utils.stage_timer import NULL_TIMER, StageTimer
from . import weights as W


@dataclass
class Layer:
    kind: str
    attn_norm: torch.Tensor
    mlp_norm: torch.Tensor
    wqkv: object = None      # bf16 tensor or ops.NvFp4Weight
    wo: object = None
    q_norm: torch.Tensor | None = None
    k_norm: torch.Tensor | None = None
    qkv_bias: torch.Tensor | None = None  # [q (| gate) | k | v] bias of this rank's heads, bf16 (attention_bias)
    dn: object = None        # DeltaNet weights
    moe: bool = False
    router_w: torch.Tensor | None = None   # [E_pad, d] bf16 (+ shared gate row)
    router_b: torch.Tensor | None = None
    w13: object = None       # NvFp4Weight (experts stacked, shared appended) or dense
    w2: object = None
    idx: tuple | None = None      # DSA indexer: (W [q|k|gate|w] bf16 padded, k_norm w, b, ape) fp32
    mla: tuple | None = None      # MLA: (W_qa, qa_norm, W_qb, W_kva, kva_norm, W_k [H,nope,512], W_v^T [H,512,v])
    hc_attn: tuple | None = None  # mHC mixing around the attention / MLP sub-layers:
    hc_mlp: tuple | None = None   # (W_mix [128 padded, hc*d] bf16, base f32, scale f32)


@dataclass
class Meta:
    """Device int32 metadata of one pass over a batch (rows = tokens)."""
    ids: torch.Tensor
    pos: torch.Tensor
    slots: torch.Tensor
    q_start: torch.Tensor
    q_len: torch.Tensor
    kv_len: torch.Tensor
    w_seq: torch.Tensor
    w_tok0: torch.Tensor
    num_work: torch.Tensor
    state_slot: torch.Tensor


@dataclass
class MtpBlock:
    """Multi-token-prediction head: [enorm(embed(t+1)) | hnorm(h_t)] -> eh_proj -> one
    attention + MoE block -> norm -> the shared lm_head."""
    enorm: torch.Tensor
    hnorm: torch.Tensor
    we: torch.Tensor        # [d, d] bf16: eh_proj columns of the embedding half
    wh: torch.Tensor        # [d, d] bf16: eh_proj columns of the hidden half
    layer: Layer
    norm: torch.Tensor
    wtap: torch.Tensor | None = None  # [d, n_taps*d] bf16: merges the tapped hidden states (mtp_taps)


def _lin_nbytes(w):
    return w.nbytes() if isinstance(w, (ops.NvFp4Weight, ops.Fp8Weight)) else w.numel() * w.element_size()


class MoELM:
    def __init__(self, cfg: ModelConfig, par: ParallelCtx | None = None, max_tokens: int = 8192,
                 max_seqs: int = 256, max_decode: int = 256, page_size: int = 64, spec_tokens: int = 0,
                 expert_order: list[int] | None = None, kv_dtype: str = "bf16"):
        self.cfg = cfg
        if kv_dtype not in ("bf16", "fp8"):
            raise ValueError("kv_dtype must be bf16 or fp8")
        if kv_dtype == "fp8" and cfg.head_dim > 128:
            raise ValueError("fp8 KV cache supports head_dim <= 128")
        if kv_dtype == "fp8" and cfg.sparse_attention is not None:
            raise ValueError("sparse (DSA) attention runs on a bf16 KV cache")
        self.kv_dtype = kv_dtype
        self.kv_torch_dtype = torch.float8_e4m3fn if kv_dtype == "fp8" else torch.bfloat16
        # expert placement: router index j serves expert expert_order[j]; rank r owns router
        # indices [r*E_l, (r+1)*E_l) (parallel/expert_balance.py builds balanced orders)
        if expert_order is not None and sorted(expert_order) != list(range(cfg.num_experts)):
            raise ValueError("expert_order must be a permutation of the experts")
        self.expert_order = list(expert_order) if expert_order is not None else list(range(cfg.num_experts))
        self.spec_k = spec_tokens
        # speculative steps draft with the MTP head when the model has one; without it the
        # drafts come from the host (engine/drafts.py) and a step only verifies them
        self.has_mtp = bool(spec_tokens and cfg.mtp_layers)
        self.mtp: MtpBlock | None = None
        self.par = par or ParallelCtx(device=torch.device("cuda", torch.cuda.current_device()))
        self.dev = self.par.device
        self.max_tokens = max_tokens
        self.max_seqs = max_seqs
        self.max_decode = max_decode
        self.page_size = page_size
        c = cfg
        tp = self.par.tp
        if c.num_q_heads % tp or c.num_kv_heads % tp:
            raise ValueError(f"heads ({c.num_q_heads}/{c.num_kv_heads}) must divide TP={tp}")
        self.Hq = c.num_q_heads // tp
        self.Hkv = c.num_kv_heads // tp
        self.E_l = c.num_experts // self.par.ep if c.num_experts else 0
        if c.num_experts and c.num_experts % self.par.ep:
            raise ValueError("experts must divide EP")
        self.e_lo = self.par.ep_rank * self.E_l
        self.shared_local = self.par.ep_rank == 0
        self.n_sh_local = c.num_shared_experts if self.shared_local else 0
        self.V_l = -(-c.vocab_size // tp)
        self.V_l = (self.V_l + 127) // 128 * 128
        self.v_lo = self.par.tp_rank * self.V_l
        self.layers: list[Layer] = []
        self.k_cache = self.v_cache = None
        self.num_pages = 0
        self.inv_freq = ops.rope_inv_freq(c.rotary_dim, c.rope_theta, self.dev)
        # ROCKET_NVTX=1: NVTX ranges around every stage (for an external timeline profiler)
        self.timer = StageTimer(False, nvtx=True) if os.environ.get("ROCKET_NVTX") else NULL_TIMER
        self.sp = None  # sequence-parallel fused decode path (set by the engine when world > 1)
        self.ar = None  # replicated-token fused path (models/ar_decode.py; set by the engine)
        self.telemetry = None  # utils.telemetry.Telemetry while attached (eager passes only)
        # act_tap(layer, site, act, T, plan): called after every NVFP4 activation quantization
        # of an eager pass (numerics tests hand the GPU's own codes to the CPU oracle)
        self.act_tap = None
        self.streamer = None  # models.expert_stream.ExpertStreamer when routed experts stream from the host
        # debug: NaN-fill the expert GEMM outputs before each MoE layer and check afterwards
        # that every routed row was written (eager steps only: the check reads back)
        self.sentinel = os.environ.get("ROCKET_SENTINEL", "0") == "1"
        self._alloc_buffers()

    # ------------------------------------------------------------------ buffers
    def _alloc_buffers(self):
        c, dev = self.cfg, self.dev
        T, S = self.max_tokens, self.max_seqs
        i32 = dict(dtype=torch.int32, device=dev)
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.ids = torch.zeros(T, **i32)
        self.pos = torch.zeros(T, **i32)
        self.slots = torch.zeros(T, **i32)
        self.q_start = torch.zeros(S, **i32)
        self.state_slot = torch.zeros(S, **i32)
        self.q_len = torch.zeros(S, **i32)
        self.kv_len = torch.zeros(S, **i32)
        self.max_pages = 0
        self.block_table = None
        G = max(1, self.Hq // max(self.Hkv, 1))
        self.max_work = S + T // max(1, 128 // G) + 1
        self.w_seq = torch.zeros(self.max_work, **i32)
        self.w_tok0 = torch.zeros(self.max_work, **i32)
        self.num_work = torch.zeros(1, **i32)
        K = self.spec_k
        # sampled rows per step: one per sequence, or every verify row under speculation
        self.max_out = min(T, S * (K + 1)) if K else S
        self.out_rows = torch.zeros(self.max_out, dtype=torch.int64, device=dev)
        # packed step outputs (one device->host copy): target ids | accepted counts | drafts [K][S]
        self.step_out = torch.zeros(self.max_out + (S + K * S if K else 0), **i32)
        self.out_ids = self.step_out[:self.max_out]
        self.keys = torch.zeros(max(self.max_out, S), dtype=torch.int64, device=dev)
        d = c.d_model
        self.x = torch.zeros(T, d, **bf)
        self.xn = torch.zeros(T, d, **bf)
        self.x_last = torch.zeros(max(self.max_out, S), d, **bf)
        if K:
            mo = self.max_out
            self.n_acc = self.step_out[mo:mo + S]
            self.drafts = self.step_out[mo + S:].view(K, S)
            self.mtp_ids = torch.zeros(T, **i32)
            self.mtp_rows = torch.zeros(S, dtype=torch.int64, device=dev)
            self.d_pos = torch.zeros(max(K - 1, 1), S, **i32)
            self.d_slots = torch.zeros(max(K - 1, 1), S, **i32)
            self.d_kvlen = torch.zeros(max(K - 1, 1), S, **i32)
            self.e_buf = torch.zeros(T, d, **bf)
            self.h_d = torch.zeros(S, d, **bf)
            # hidden-tap drafting: residual stream after each tapped layer, [T, n_taps * d]
            self.tap_slot = {li: k for k, li in enumerate(c.mtp_taps)} if self.has_mtp else {}
            if self.tap_slot:
                if c.hc_streams:
                    raise ValueError("mtp_taps: the draft taps read one residual stream (no hyper-connections)")
                if any(not 0 <= li < c.num_layers for li in c.mtp_taps):
                    raise ValueError(f"mtp_taps {c.mtp_taps} outside the {c.num_layers} layers")
                self.taps = torch.zeros(T, len(c.mtp_taps) * d, **bf)
                self.tap_h = torch.zeros(T, d, **bf)
            self.d_arange = torch.arange(S, **i32)
            self.d_ones = torch.ones(S, **i32)
            self.d_zeros = torch.zeros(S, **i32)
            self.d_nwork = torch.zeros(1, **i32)
            # per-step host-staged flags (bound into the engine's packed metadata)
            self.verify = torch.zeros(S, **i32)
            self.sample = torch.zeros(S, **i32)
            self.out_idx = torch.zeros(T, **i32)
            self.next_tok = torch.zeros(T, **i32)
        qd = self.Hq * c.head_dim
        self.qkv_dim = (qd * (2 if c.attn_output_gate else 1)) + 2 * self.Hkv * c.head_dim
        self.qkv = torch.zeros(T, self.qkv_dim, **bf)
        self.q = torch.zeros(T, self.Hq, c.head_dim, **bf)
        self.gate = torch.zeros(T, self.Hq, c.head_dim, **bf) if c.attn_output_gate else None
        self.attn_out = torch.zeros(T, qd, **bf)
        self.splits = 1   # attention key splits of decode steps (one row per sequence)
        self.vsplits = 1  # ... of speculative verify passes (K+1 rows per sequence)
        self.ws_o = self.ws_ml = None
        fa = c.weight_format.get("attention", "bf16")
        act = ops.NvFp4Act if fa == "nvfp4" else (ops.Fp8Act if fa == "fp8" else None)
        self.xq_attn = act(T, d, dev) if act else None
        self.xq_attn_o = act(T, qd, dev) if act else None
        self.xq_head = ops.NvFp4Act(S, d, dev) if c.weight_format.get("lm_head", "bf16") == "nvfp4" else None
        if c.num_experts:
            k_out = c.top_k + c.num_shared_experts
            e_tot = self.E_l + c.num_shared_experts
            # small-batch plan (32-token tiles): decode steps and speculative verify passes
            self.plan_dec_tokens = min(T, self.max_decode * (self.spec_k + 1))
            self.plan_dec = ops.MoePlan(self.plan_dec_tokens, k_out, e_tot, 32, dev)
            self.k_out, self.e_tot = k_out, e_tot
            self.plan_pre = ops.MoePlan(T, k_out, e_tot, 128, dev)
            rows = max(self.plan_dec.max_rows, self.plan_pre.max_rows)
            self.xq = ops.NvFp4Act(rows, d, dev)
            inter = c.moe_intermediate
            self.h = torch.zeros(rows, inter, **bf)
            self.hq = ops.NvFp4Act(rows, inter, dev)
            self.y = torch.zeros(rows, d, **bf)
            self.E_pad = (c.num_experts + (1 if c.shared_expert_gate else 0) + 127) // 128 * 128
            self.logits = torch.zeros(T, self.E_pad, dtype=torch.float32, device=dev)
        if c.num_dense_layers:
            I_l = c.dense_intermediate // self.par.tp
            self.hd = torch.zeros(T, I_l, **bf)
            self.xq_d = ops.NvFp4Act(T, d, dev)
            self.hq_d = ops.NvFp4Act(T, I_l, dev)
        if c.mla is not None:
            ml = c.mla
            self.mla_rows = min(T, 1024)  # MLA scratch rows (longer passes run in row chunks)
            f32 = dict(dtype=torch.float32, device=dev)
            self.q_lat = torch.zeros(T, ml.q_lora_rank, **bf)
            self.q_lat_n = torch.zeros(T, ml.q_lora_rank, **bf)
            self.q_nope = torch.zeros(T, (self.Hq * ml.qk_nope_head_dim + 127) // 128 * 128, **bf)
            self.kv_lat = torch.zeros(T, ml.kv_lora_rank, **bf)
            self.mla_qabs = torch.zeros(self.mla_rows, self.Hq, ml.kv_lora_rank, **f32)
            self.mla_ctx = torch.zeros(self.mla_rows, self.Hq, ml.kv_lora_rank, **f32)
        sa = c.sparse_attention
        if sa is not None:
            self.idx_cols = sa.index_heads * sa.index_dim + 2 * sa.index_dim + sa.index_heads
            self.idx_proj = torch.zeros(T, (self.idx_cols + 127) // 128 * 128, **bf)
            self.dsa_sel = torch.zeros(T, sa.top_k + sa.kpool - 1, dtype=torch.int32, device=dev)
            self.dsa_nsel = torch.zeros(T, dtype=torch.int32, device=dev)
        self.hc = c.hc_streams
        if self.hc:
            hc = self.hc
            self.streams = torch.zeros(T, hc, d, **bf)       # hyper-connection residual streams
            self.hc_mix = torch.zeros(T, 128, dtype=torch.float32, device=dev)
            self.hc_coef = torch.zeros(T, hc + hc * hc, dtype=torch.float32, device=dev)
        if any(c.layer_kind(i) == "deltanet" for i in range(c.num_layers)):
            from .deltanet import DeltaNetBuffers
            # +1: scratch slot of padded rows; verify rows of a speculative step are retained
            self.dn_buf = DeltaNetBuffers(c, self.par, T, S + 1, dev, spec_rows=self.max_out if self.spec_k else 0)

    def allocate_kv(self, num_pages: int, max_pages_per_seq: int):
        c = self.cfg
        n_attn = sum(1 for i in range(c.num_layers) if c.layer_kind(i) == "attention")
        self.attn_index = {}
        j = 0
        for i in range(c.num_layers):
            if c.layer_kind(i) == "attention":
                self.attn_index[i] = j
                j += 1
        if self.has_mtp:
            self.attn_index["mtp"] = j  # the MTP head's attention keeps its own KV in the same pages
            n_attn += 1
        ps = self.page_size
        kd = self.kv_torch_dtype
        if c.mla is not None:
            # MLA caches one latent row per token (stored as the K cache with one 512-wide
            # "head"); there is no separate V cache
            self.k_cache = torch.zeros(n_attn, num_pages, 1, ps, c.mla.kv_lora_rank, dtype=kd, device=self.dev)
            self.v_cache = torch.zeros(n_attn, num_pages, 1, 0, ps, dtype=kd, device=self.dev)
        else:
            self.k_cache = torch.zeros(n_attn, num_pages, self.Hkv, ps, c.head_dim, dtype=kd, device=self.dev)
            self.v_cache = torch.zeros(n_attn, num_pages, self.Hkv, c.head_dim, ps, dtype=kd, device=self.dev)
        # fp8 caches store value / scale (per attention layer; 1.0 unless calibrated)
        self.k_scales = [1.0] * n_attn
        self.v_scales = [1.0] * n_attn
        self.num_pages = num_pages
        self.max_pages = max_pages_per_seq
        self.block_table = torch.zeros(self.max_seqs, max_pages_per_seq, dtype=torch.int32, device=self.dev)
        sa = c.sparse_attention
        if sa is not None:
            # per-token indexer keys and compressor gates (same pages as K/V) and pool-score scratch
            bf = dict(dtype=torch.bfloat16, device=self.dev)
            self.ik_cache = torch.zeros(n_attn, num_pages * ps, sa.index_dim, **bf)
            self.ig_cache = torch.zeros(n_attn, num_pages * ps, sa.index_dim, **bf)
            self.dsa_scores = torch.zeros(self.max_tokens, max(1, max_pages_per_seq * ps // sa.kpool),
                                          dtype=torch.float32, device=self.dev)

    def page_caches(self) -> list:
        """Every per-page device cache as a [layers, pages, ...] view: K, V (and the DSA index
        keys / gates).  Page-granular tiers (prefix store, session checkpoints) copy these."""
        out = [self.k_cache, self.v_cache]
        if self.cfg.sparse_attention is not None:
            L = self.ik_cache.shape[0]
            for t in (self.ik_cache, self.ig_cache):
                out.append(t.view(L, self.num_pages, self.page_size, t.shape[-1]))
        return out

    def kv_bytes_per_page(self) -> int:
        c = self.cfg
        n_attn = sum(1 for i in range(c.num_layers) if c.layer_kind(i) == "attention") + (1 if self.has_mtp else 0)
        if c.mla is not None:
            kv = n_attn * self.page_size * c.mla.kv_lora_rank * 2
        else:
            kv = n_attn * 2 * self.Hkv * self.page_size * c.head_dim * (1 if self.kv_dtype == "fp8" else 2)
        if c.sparse_attention is not None:
            kv += n_attn * 2 * self.page_size * c.sparse_attention.index_dim * 2
        return kv

    def auto_decode_splits(self, batch: int, ctx: int, max_splits: int = 8) -> int:
        """Key splits for attention of `batch` single-block work items so (batch x kv heads
        x splits) CTAs fill whole waves of SMs (one CTA per SM) without splitting below 2
        key blocks of 128.  Small batches may split further (up to `max_splits`)."""
        items = batch * self.Hkv
        sms = ops.num_sms()
        max_s = max(1, min(max_splits, ctx // 256))
        best, best_eff = 1, 0.0
        for s in range(1, max_s + 1):
            n = items * s
            eff = n / (-(-n // sms) * sms) - 0.01 * (s - 1)
            if eff > best_eff:
                best, best_eff = s, eff
        return best

    def configure_attention(self, batch: int, ctx: int):
        """Split-K choice for the captured step shapes at context `ctx`: decode rows (one
        per sequence) and speculative verify rows (K+1 per sequence), and one workspace
        sized for the larger of the two."""
        max_s = 64 if batch * self.Hkv < 32 else 8  # very small batches split deeper
        self.splits = self.auto_decode_splits(batch, ctx, max_s)
        self.vsplits = self.auto_decode_splits(batch, ctx, max_s) if self.spec_k else 1
        rows = max(self.splits * self.max_seqs, self.vsplits * self.max_out)
        if max(self.splits, self.vsplits) > 1:
            n = rows * self.Hq
            self.ws_o = torch.empty(n * self.cfg.head_dim, dtype=torch.float32, device=self.dev)
            self.ws_ml = torch.empty(n * 2, dtype=torch.float32, device=self.dev)

    def set_decode_splits(self, splits: int, max_rows: int):
        if splits > 1:
            self.ws_o = torch.empty(splits, max_rows * self.Hq, self.cfg.head_dim, dtype=torch.float32, device=self.dev)
            self.ws_ml = torch.empty(splits, max_rows * self.Hq, 2, dtype=torch.float32, device=self.dev)
        self.splits = splits

    def weight_bytes(self) -> int:
        n = self.embed.numel() * 2 + _lin_nbytes(self.lm_head)
        for L in self.layers:
            for w in (L.wqkv, L.wo, L.w13, L.w2, L.router_w):
                if w is not None:
                    n += _lin_nbytes(w)
            if L.dn is not None:
                n += L.dn.nbytes()
        if self.mtp is not None:
            M = self.mtp
            n += (M.we.numel() + M.wh.numel()) * 2
            for w in (M.layer.wqkv, M.layer.wo, M.layer.w13, M.layer.w2, M.layer.router_w):
                if w is not None:
                    n += _lin_nbytes(w)
        return n

    # ------------------------------------------------------------------ weights
    def enable_expert_streaming(self, slots: int):
        """Keep routed experts in pinned host memory with `slots` device slots per MoE
        layer (models/expert_stream.py); call before the weights are built.  Eager
        execution only (each MoE layer reads its routing back to the host)."""
        from .expert_stream import ExpertStreamer
        if not self.cfg.num_experts:
            raise ValueError("expert streaming needs a MoE model")
        self.streamer = ExpertStreamer(self.E_l, self.cfg.num_shared_experts, slots, self.dev)

    def _stream(self, L):
        if self.streamer is not None and getattr(L, "moe", False):
            self.streamer.adopt(L)
        return L

    def load_fuel(self, t: dict, expert_slab: str | None = None):
        """Shard and convert fuel-format tensors (CPU) into the engine layout.  With
        `expert_slab` (this rank's slab, fuel/slabs.py) the routed and shared experts are
        read from the slab instead of `t`, which then needs no expert tensors."""
        c, dev = self.cfg, self.dev
        if expert_slab and self.streamer is not None:
            raise ValueError("expert streaming reads experts from the fuel tensors, not from a slab")
        self._slab_w = {} if expert_slab else None
        self.layers = []
        v0, v1 = self.v_lo, min(c.vocab_size, self.v_lo + self.V_l)
        # the embedding table is replicated: any rank embeds any token without a collective
        self.embed = t["embed.weight"].to(dev)
        for i in range(c.num_layers):
            self.layers.append(self._stream(self._load_block(t, f"layers.{i}", c.layer_kind(i), c.is_moe_layer(i))))
        self.final_norm = t["final_norm.weight"].to(dev)
        lm = self._rows(t, "lm_head", v0, v1)
        self.lm_head = self._cat_lin([lm], pad=True, pad_to=self.V_l)
        if self.has_mtp:
            pre = "mtp.0"
            eh = W.dequant(t, f"{pre}.eh_proj").bfloat16()  # bf16 on the GPU (either fuel format)
            d = c.d_model
            self.mtp = MtpBlock(t[f"{pre}.enorm.weight"].to(dev), t[f"{pre}.hnorm.weight"].to(dev),
                                eh[:, :d].contiguous().to(dev), eh[:, d:].contiguous().to(dev),
                                self._stream(self._load_block(t, f"{pre}.layer", "attention", c.num_experts > 0)),
                                t[f"{pre}.norm.weight"].to(dev))
            if c.mtp_taps:
                self.mtp.wtap = W.dequant(t, f"{pre}.tap_proj").bfloat16().contiguous().to(dev)
        if expert_slab:
            self._read_expert_slab(expert_slab)

    def _read_expert_slab(self, path: str):
        from ..fuel import slabs
        hdr = slabs.read_header(path)
        par = self.par
        if (hdr["rank"], hdr["world"]) != (par.ep_rank, par.ep):
            raise ValueError(f"{path}: slab of EP rank {hdr['rank']}/{hdr['world']}, this is {par.ep_rank}/{par.ep}")
        if hdr["expert_order"] != list(self.expert_order):
            raise ValueError(f"{path}: slab packed for a different expert order")
        have = {L["prefix"]: [s["name"] for s in L["slots"]] for L in hdr["layers"]}
        for pre, (_, _, names) in self._slab_w.items():
            if have.get(pre) != names:
                raise ValueError(f"{path}: layer {pre}: slab slots do not match this rank's experts")
        tg = slabs.engine_targets({pre: (w13, w2) for pre, (w13, w2, _) in self._slab_w.items()})
        self.slab_stats = slabs.read_slab(path, tg)
        self._slab_w = None

    def _load_block(self, t: dict, pre: str, kind: str, is_moe: bool) -> Layer:
        c, dev, par = self.cfg, self.dev, self.par
        D = c.head_dim
        L = Layer(kind=kind, attn_norm=t[f"{pre}.attn_norm.weight"].to(dev),
                  mlp_norm=t[f"{pre}.mlp_norm.weight"].to(dev))
        if f"{pre}.hc_attn.fn" in t:
            L.hc_attn, L.hc_mlp = (self._hc_weights(t[f"{pre}.{s}.fn"], t[f"{pre}.{s}.base"], t[f"{pre}.{s}.scale"])
                                   for s in ("hc_attn", "hc_mlp"))
        if L.kind == "attention" and c.mla is not None:
            L.mla, L.wo = self._load_mla(t, pre)
        elif L.kind == "attention":
            q0, q1 = par.tp_rank * self.Hq * D, (par.tp_rank + 1) * self.Hq * D
            k0, k1 = par.tp_rank * self.Hkv * D, (par.tp_rank + 1) * self.Hkv * D
            parts = []
            qn = f"{pre}.attn.q_proj"
            parts.append(self._rows(t, qn, q0, q1))
            if c.attn_output_gate:
                parts.append(self._rows(t, qn, c.q_dim + q0, c.q_dim + q1))
            parts.append(self._rows(t, f"{pre}.attn.k_proj", k0, k1))
            parts.append(self._rows(t, f"{pre}.attn.v_proj", k0, k1))
            L.wqkv = self._attn_fmt(self._cat_lin(parts, pad=True))
            if c.attention_bias:
                qb, kb, vb = (t[f"{pre}.attn.{n}.bias"] for n in ("q_proj", "k_proj", "v_proj"))
                bs = [qb[q0:q1]] + ([qb[c.q_dim + q0:c.q_dim + q1]] if c.attn_output_gate else [])
                L.qkv_bias = torch.cat(bs + [kb[k0:k1], vb[k0:k1]]).bfloat16().to(dev)
            L.wo = self._attn_fmt(self._cat_lin([self._cols(t, f"{pre}.attn.o_proj", q0, q1)]))
            if c.qk_norm:
                L.q_norm = t[f"{pre}.attn.q_norm.weight"].to(dev)
                L.k_norm = t[f"{pre}.attn.k_norm.weight"].to(dev)
        else:
            from .deltanet import load_deltanet
            L.dn = load_deltanet(c, t, pre, par, dev, index=self._dn_count())
        if L.kind == "attention" and c.sparse_attention is not None:
            ip = f"{pre}.attn.indexer"
            w = torch.cat([W.dequant(t, f"{ip}.{n}") for n in ("wq", "wk", "wgate", "wproj")])
            L.idx = self._idx_weights(w, t[f"{ip}.k_norm.weight"], t[f"{ip}.k_norm.bias"], t[f"{ip}.ape"])
        if is_moe:
            L.moe = True
            E = c.num_experts
            order = torch.tensor(self.expert_order, dtype=torch.long)
            rw = torch.zeros(self.E_pad, c.d_model, dtype=torch.bfloat16)
            rw[:E] = t[f"{pre}.moe.router.weight"][order]
            if c.shared_expert_gate:
                rw[E] = t[f"{pre}.moe.shared_gate.weight"][0]
            L.router_w = rw.to(dev)
            if f"{pre}.moe.router.bias" in t:
                L.router_b = t[f"{pre}.moe.router.bias"].float()[order].contiguous().to(dev)
            w13s, w2s = [], []
            names = [f"{pre}.moe.experts.{self.expert_order[e]}" for e in range(self.e_lo, self.e_lo + self.E_l)]
            # every rank holds the shared experts (the sequence-parallel decode path runs them
            # for the rank's own tokens; the replicated path routes them to rank 0 only)
            names += ([f"{pre}.moe.shared"] if c.num_shared_experts == 1 else
                      [f"{pre}.moe.shared.{s}" for s in range(c.num_shared_experts)])
            if self._slab_w is not None:
                # experts come from the slab: allocate the stacked weights, fill them later
                n_e, I, d = len(names), c.moe_intermediate, c.d_model
                L.w13 = W.empty_nvfp4(2 * I, d, n_e, dev)
                L.w2 = W.empty_nvfp4(d, I, n_e, dev)
                self._slab_w[pre] = (L.w13, L.w2, names)
            else:
                for nm in names:
                    w13s.append(W.fuse_w13(W.triplet_of(t, nm + ".gate_proj"), W.triplet_of(t, nm + ".up_proj")))
                    w2s.append(W.triplet_of(t, nm + ".down_proj"))
                L.w13 = W.stack_nvfp4(w13s, dev)
                L.w2 = W.stack_nvfp4(w2s, dev)
        else:
            I0, I1 = par.shard(c.dense_intermediate, "dense intermediate")
            g = self._rows_nv(t, f"{pre}.mlp.gate_proj", I0, I1)
            u = self._rows_nv(t, f"{pre}.mlp.up_proj", I0, I1)
            L.w13 = W.stack_nvfp4([W.fuse_w13(g, u)], dev)
            L.w2 = W.stack_nvfp4([self._cols_nv(t, f"{pre}.mlp.down_proj", I0, I1)], dev)
        return L

    def _attn_fmt(self, w):
        """Attention projections in the fuel's attention format (FP8-row requantizes the
        rows from their exact values; bf16 / NVFP4 pass through)."""
        if self.cfg.weight_format.get("attention", "bf16") == "fp8" and not isinstance(w, ops.NvFp4Weight):
            return ops.Fp8Weight.quantize(w.float(), self.dev)
        return w

    def _load_mla(self, t, pre):
        """MLA weights of this rank's heads: low-rank query path, latent projection, and
        kv_b split into W_k [H, nope, 512] and W_v^T [H, 512, v]; o_proj columns."""
        c, ml, par = self.cfg, self.cfg.mla, self.par
        H, nope, v = self.Hq, ml.qk_nope_head_dim, ml.v_head_dim
        h0 = par.tp_rank * H
        a = f"{pre}.attn"
        kvb = W.dequant(t, f"{a}.kv_b_proj").view(c.num_q_heads, nope + v, ml.kv_lora_rank)[h0:h0 + H]
        qb = W.dequant(t, f"{a}.q_b_proj")[h0 * nope:(h0 + H) * nope]
        wo = W.dequant(t, f"{a}.o_proj")[:, h0 * v:(h0 + H) * v]
        return self._mla_weights(W.dequant(t, f"{a}.q_a_proj"), t[f"{a}.q_a_norm.weight"], qb,
                                 W.dequant(t, f"{a}.kv_a_proj"), t[f"{a}.kv_a_norm.weight"], kvb, wo)

    def _mla_weights(self, qa, qan, qb, kva, kvan, kvb, wo):
        nope = self.cfg.mla.qk_nope_head_dim
        dev = self.dev
        b = lambda x: x.bfloat16().contiguous().to(dev)
        pad = lambda x: W.pad_rows(x.bfloat16(), 128).contiguous().to(dev)
        return ((pad(qa), b(qan), pad(qb), pad(kva), b(kvan), b(kvb[:, :nope]),
                 b(kvb[:, nope:].transpose(1, 2))), b(wo))

    def _idx_weights(self, w, knw, knb, ape):
        """DSA indexer in the engine layout: one bf16 GEMM weight [q | k | gate | head w]
        (rows padded to 128), fp32 key-norm weight / bias and pool-slot offsets."""
        f32 = dict(dtype=torch.float32, device=self.dev)
        return (W.pad_rows(w.bfloat16(), 128).contiguous().to(self.dev), knw.to(**f32).contiguous(),
                knb.to(**f32).contiguous(), ape.to(**f32).contiguous())

    def _hc_weights(self, fn, base, scale):
        """mHC site weights in the engine layout: the mix projection padded to a 128-row
        GEMM tile, fp32 bias / scales on the device."""
        return (W.pad_rows(fn.bfloat16(), 128).contiguous().to(self.dev),
                base.float().contiguous().to(self.dev), scale.float().contiguous().to(self.dev))

    def _dn_count(self) -> int:
        return sum(1 for L in self.layers if L.dn is not None)

    def _rows(self, t, name, r0, r1):
        if t[name + ".weight"].dtype == torch.float8_e4m3fn:  # FP8-row fuel: exact fp32 rows
            return W.dequant(t, name)[r0:r1]
        if name + ".weight_scale" in t:
            return self._rows_nv(t, name, r0, r1)
        return t[name + ".weight"][r0:r1]

    def _rows_nv(self, t, name, r0, r1):
        tr = W.triplet_of(t, name)
        return W.NvTriplet(tr.packed[r0:r1], tr.sf[r0:r1], tr.gscale[r0:r1])

    def _cols(self, t, name, c0, c1):
        if t[name + ".weight"].dtype == torch.float8_e4m3fn:
            return W.dequant(t, name)[:, c0:c1]
        if name + ".weight_scale" in t:
            return self._cols_nv(t, name, c0, c1)
        return t[name + ".weight"][:, c0:c1]

    def _cols_nv(self, t, name, c0, c1):
        tr = W.triplet_of(t, name)
        assert c0 % 16 == 0 and c1 % 16 == 0
        return W.NvTriplet(tr.packed[:, c0 // 2:c1 // 2].contiguous(), tr.sf[:, c0 // 16:c1 // 16].contiguous(),
                           tr.gscale)

    def _cat_lin(self, parts, pad=False, pad_to=None):
        if isinstance(parts[0], W.NvTriplet):
            p = W.NvTriplet(torch.cat([x.packed for x in parts]), torch.cat([x.sf for x in parts]),
                            torch.cat([x.gscale for x in parts]))
            n = p.packed.shape[0]
            tgt = pad_to or ((n + 127) // 128 * 128 if pad else n)
            if tgt != n:
                p = W.NvTriplet(W.pad_rows(p.packed, tgt), W.pad_rows(p.sf, tgt),
                                torch.cat([p.gscale, torch.ones(tgt - n)]))
            return W.stack_nvfp4([p], self.dev)
        w = torch.cat(parts)
        w = w if w.dtype == torch.float32 else w.bfloat16()  # fp32: exact FP8-row values, requantized by _attn_fmt
        n = w.shape[0]
        tgt = pad_to or ((n + 127) // 128 * 128 if pad else n)
        return W.pad_rows(w, tgt).contiguous().to(self.dev)

    def init_random(self, seed: int = 0):
        """Random N(0, init_std) weights generated directly on the GPU in the engine
        layout (the benchmark serving configs use random-init weights of the real shape)."""
        c, dev, par = self.cfg, self.dev, self.par
        std = c.init_std
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed * 1000003 + par.rank)  # sharded tensors: per-rank stream
        gen_rep = torch.Generator(device=dev)
        gen_rep.manual_seed(seed * 1000003 + 7919)  # replicated tensors: identical on every rank
        # tensor-parallel tensors (attention, dense MLP, vocab) and routed experts are per-rank
        # streams only when that dimension is split; replicated layouts (tp = 1 or ep = 1 on
        # several ranks) must hold the same weights on every rank
        gen_tp = gen if par.tp > 1 else gen_rep
        gen_ep = gen if par.ep > 1 else gen_rep
        bf = dict(dtype=torch.bfloat16, device=dev)
        d, D = c.d_model, c.head_dim

        def rnd(n, k):
            return (torch.randn(n, k, generator=gen_tp, **bf) * std)

        def lin(n, k, fmt, pad=True):
            n_pad = (n + 127) // 128 * 128 if pad else n
            if fmt == "nvfp4":
                return W.random_nvfp4_on_device((n_pad, k), 1, std, gen_tp, dev)
            if fmt == "fp8":
                w = torch.zeros(n_pad, k, **bf)
                w[:n] = rnd(n, k)
                return ops.Fp8Weight.quantize(w)
            w = torch.zeros(n_pad, k, **bf)
            w[:n] = rnd(n, k)
            return w

        one = (lambda n: torch.zeros(n, **bf)) if c.zero_centered_norm else (lambda n: torch.ones(n, **bf))
        self.embed = torch.randn(c.vocab_size, d, generator=gen_rep, **bf) * std  # replicated
        fa = c.weight_format.get("attention", "bf16")

        def block(kind, is_moe, hc=False):
            L = Layer(kind=kind, attn_norm=one(d), mlp_norm=one(d))
            if kind == "attention" and c.mla is not None:
                ml = c.mla
                r = lambda n, k: torch.randn(n, k, generator=gen_tp, **bf) * std       # this rank's heads
                rr = lambda n, k: torch.randn(n, k, generator=gen_rep, **bf) * std     # replicated
                H, nope, v = self.Hq, ml.qk_nope_head_dim, ml.v_head_dim
                L.mla, L.wo = self._mla_weights(rr(ml.q_lora_rank, d), torch.ones(ml.q_lora_rank),
                                                r(H * nope, ml.q_lora_rank), rr(ml.kv_lora_rank, d),
                                                torch.ones(ml.kv_lora_rank),
                                                r(H * (nope + v), ml.kv_lora_rank).view(H, nope + v, -1),
                                                r(d, H * v))
                kind = "mla"
            if hc:
                nm = 2 * c.hc_streams + c.hc_streams ** 2
                L.hc_attn, L.hc_mlp = (self._hc_weights(
                    torch.randn(nm, c.hc_streams * d, generator=gen_rep, **bf) * std,
                    torch.randn(nm, generator=gen_rep, device=dev) * 0.5, torch.ones(3)) for _ in range(2))
            if kind == "mla":
                pass
            elif L.kind == "attention":
                L.wqkv = lin(self.qkv_dim, d, fa)
                if c.attention_bias:
                    L.qkv_bias = (torch.randn(self.qkv_dim, generator=gen_tp, device=dev) * 0.5).bfloat16()
                L.wo = lin(d, self.Hq * D, fa)
                if c.qk_norm:
                    L.q_norm, L.k_norm = one(D), one(D)
            else:
                from .deltanet import random_deltanet
                L.dn = random_deltanet(c, par, gen_tp, dev, index=self._dn_count())
            sa = c.sparse_attention
            if sa is not None and L.kind == "attention":  # the indexer is replicated on every rank
                L.idx = self._idx_weights(torch.randn(self.idx_cols, d, generator=gen_rep, **bf) * std,
                                          torch.ones(sa.index_dim), torch.zeros(sa.index_dim),
                                          torch.randn(sa.kpool, sa.index_dim, generator=gen_rep, device=dev) * 0.5)
            if is_moe:
                L.moe = True
                L.router_w = torch.zeros(self.E_pad, d, **bf)
                ne_r = c.num_experts + (1 if c.shared_expert_gate else 0)
                L.router_w[:ne_r] = torch.randn(ne_r, d, generator=gen_rep, **bf) * std
                if c.router == "sigmoid":
                    L.router_b = torch.zeros(c.num_experts, dtype=torch.float32, device=dev)
                ne = self.E_l + c.num_shared_experts  # shared experts replicated on every rank
                L.w13 = W.random_nvfp4_on_device((2 * c.moe_intermediate, d), ne, std, gen_ep, dev,
                                                 fuse_swiglu=True)
                L.w2 = W.random_nvfp4_on_device((d, c.moe_intermediate), ne, std, gen_ep, dev)
                if c.num_shared_experts and par.ep > 1:
                    # identical shared experts on every rank (any rank may own them per layer)
                    sh13 = W.random_nvfp4_on_device((2 * c.moe_intermediate, d), c.num_shared_experts, std,
                                                    gen_rep, dev, fuse_swiglu=True)
                    sh2 = W.random_nvfp4_on_device((d, c.moe_intermediate), c.num_shared_experts, std, gen_rep, dev)
                    W.set_expert_tail(L.w13, sh13)
                    W.set_expert_tail(L.w2, sh2)
            else:
                I_l = c.dense_intermediate // par.tp
                L.w13 = W.random_nvfp4_on_device((2 * I_l, d), 1, std, gen_tp, dev, fuse_swiglu=True)
                L.w2 = W.random_nvfp4_on_device((d, I_l), 1, std, gen_tp, dev)
            return L

        self.layers = []
        for i in range(c.num_layers):
            self.layers.append(self._stream(block(c.layer_kind(i), c.is_moe_layer(i), hc=c.hc_streams > 0)))
        self.final_norm = one(d)
        self.lm_head = lin(self.V_l, d, c.weight_format.get("lm_head", "bf16"), pad=False)
        if self.has_mtp:
            # eh_proj is replicated (every rank embeds and projects all rows)
            eh = torch.randn(d, 2 * d, generator=gen_rep, **bf) * std
            self.mtp = MtpBlock(one(d), one(d), eh[:, :d].contiguous(), eh[:, d:].contiguous(),
                                self._stream(block("attention", c.num_experts > 0)), one(d))
            if c.mtp_taps:
                self.mtp.wtap = torch.randn(d, len(c.mtp_taps) * d, generator=gen_rep, **bf) * std
        torch.cuda.synchronize(dev)

    # ------------------------------------------------------------------ forward
    def _linear(self, x, w, out, epi=ops.EPI_STORE_BF16, residual=None, T=None, xq=None, fused=None):
        T = x.shape[0] if T is None else T
        if isinstance(w, ops.Fp8Weight):
            ops.quantize_rows_fp8(x, xq, T)
            return ops.linear_fp8(xq, T, w, out=out, epi=epi, residual=residual, fused=fused)
        if isinstance(w, ops.NvFp4Weight):
            ops.quantize_rows(x, xq, T)
            return ops.linear_nvfp4(xq, T, w, out=out, epi=epi, residual=residual, fused=fused)
        return ops.linear_bf16(x, w, out=out, epi=epi, residual=residual, fused=fused)

    def _norm_into_xn(self, w, T):
        """`fused` entries that make a residual GEMM also write RMSNorm(x) * w into xn."""
        c = self.cfg
        return ops.norm_args(w, self.xn[:T], c.norm_eps, c.zero_centered_norm)

    def main_meta(self) -> Meta:
        """Metadata of the step staged by the engine (its packed int32 buffer)."""
        return Meta(self.ids, self.pos, self.slots, self.q_start, self.q_len, self.kv_len, self.w_seq, self.w_tok0,
                    self.num_work, self.state_slot)

    def forward(self, T: int, S: int, W_: int, n_out: int, decode: bool, logits_out=None) -> torch.Tensor:
        if decode and logits_out is None and getattr(self, "sp", None) is not None and self.sp.handles(T, n_out):
            return self.sp.forward(T, W_)
        ar = getattr(self, "ar", None)
        if ar is not None and (decode or ar.tp == 1) and ar.handles(T, n_out):
            return ar.forward(T, S, W_, n_out, decode, logits_out)
        return self.forward_replicated(T, S, W_, n_out, decode, logits_out)

    def forward_replicated(self, T: int, S: int, W_: int, n_out: int, decode: bool, logits_out=None,
                           spec_rows: int = 0) -> torch.Tensor:
        """One engine step over the batch already staged in the static buffers.

        T tokens (ids/pos/slots), S sequences (q_start/q_len/kv_len/block_table),
        W_ attention work items, n_out rows to sample (out_rows).  Returns out_ids[:n_out].
        `spec_rows`: rows [0, spec_rows) are speculative verify rows (DeltaNet layers keep
        their state for the commit).  The last-layer hidden states stay in self.x[:T].
        """
        meta = self.main_meta()
        x = self.x[:T]
        tm = self.timer
        tm.start("embed")
        ops.embed(meta.ids[:T], self.embed, x, 0)
        if self.hc:
            ops.hc_expand(self.hc, self.streams[:T], x, T)
        tm.stop("embed")
        self._prenormed = False
        for i, L in enumerate(self.layers):
            self._block(L, i, x, T, S, W_, decode, meta, spec_rows)
            self.capture_tap(i, x, T)
        if self.hc:
            ops.hc_mean(self.hc, self.streams[:T], x, T)  # the head reads the mean of the streams
        tm.start("lm_head")
        # sampled rows -> final norm -> lm_head with fused argmax (vocab-parallel)
        xs = torch.index_select(x, 0, self.out_rows[:n_out], out=self.x_last[:n_out])
        out = self._head(xs, n_out, self.final_norm, self.out_ids[:n_out], logits_out)
        tm.stop("lm_head")
        return out

    def _block(self, L, i, x, T, S, W_, decode, meta: Meta, spec_rows: int = 0):
        """One decoder block (attention or DeltaNet, then MoE or dense MLP) in place on x."""
        c, par, tm = self.cfg, self.par, self.timer
        self._cur_layer = i
        self._n_seqs = S  # sequences of this pass (sparse attention maps rows to sequences)
        lead = par.tp_rank == 0  # the rank that adds the residual before a partial-sum all-reduce
        hc = L.hc_attn is not None
        if hc:
            # x := mixed sub-layer input; the sub-layer then writes its output y into x
            # (no residual add) and the combine folds y into the streams
            self._hc_split(L.hc_attn, x, T)
            lead = False
        if getattr(self, "_prenormed", False):
            xn = self.xn[:T]  # the previous block's last kernel wrote this block's attention norm
        else:
            tm.start("norm")
            xn = ops.rmsnorm(x, L.attn_norm, c.norm_eps, c.zero_centered_norm, out=self.xn[:T])
            tm.stop("norm")
        self._prenormed = False
        # with no collective between them, a sub-layer's residual kernel also writes the next
        # norm (x and xn exactly as the two kernels would)
        single = par.tp == 1 and par.ep == 1 and not self.hc
        if L.kind == "attention":
            post = L.mlp_norm if (single and L.mla is None) else None
            self._attention(i, L, xn, x, T, W_, decode, lead, meta, post_norm=post)
        else:
            from .deltanet import deltanet_forward
            tm.start("deltanet")
            deltanet_forward(self, i, L, xn, x, T, S, decode, lead, meta, spec_rows)
            tm.stop("deltanet")
        if par.tp > 1:
            tm.start("allreduce")
            par.all_reduce(x)
            tm.stop("allreduce")
        if hc:
            ops.hc_combine(self.hc, self.streams[:T], x, self.hc_coef[:T], T)
            self._hc_split(L.hc_mlp, x, T)
        if L.kind == "attention" and post is not None:
            xn = self.xn[:T]
        else:
            tm.start("norm")
            xn = ops.rmsnorm(x, L.mlp_norm, c.norm_eps, c.zero_centered_norm, out=self.xn[:T])
            tm.stop("norm")
        # the MLP's partial sums span the expert-parallel group (MoE) or the tensor-parallel
        # group (dense); its residual is added by that group's first rank
        mlp_group = par.ep if L.moe else par.tp
        mlp_lead = (par.ep_rank == 0 if L.moe else par.tp_rank == 0) and not hc
        # the next decoder block's attention norm (not after the last block or an MTP block)
        nxt = self.layers[i + 1].attn_norm if (single and isinstance(i, int) and i + 1 < len(self.layers)) else None
        if L.moe:
            self._prenormed = self._moe(L, xn, x, T, decode, mlp_lead, next_norm=nxt)
        else:
            tm.start("dense_mlp")
            self._prenormed = self._dense(L, xn, x, T, mlp_lead, next_norm=nxt)
            tm.stop("dense_mlp")
        if mlp_group > 1:
            tm.start("allreduce")
            par.all_reduce(x)
            tm.stop("allreduce")
        if hc:
            ops.hc_combine(self.hc, self.streams[:T], x, self.hc_coef[:T], T)
        if self.telemetry is not None:
            self.telemetry.layer(i, x)

    def _hc_split(self, site, x, T):
        """x[:T] := sum_i pre_i * stream_i for one mHC site (mix GEMM on the raw streams,
        then coefficients + Sinkhorn + collapse in one kernel)."""
        c, tm = self.cfg, self.timer
        fn, base, scale = site
        tm.start("hyper_connection")
        flat = self.streams[:T].view(T, -1)
        ops.linear_bf16(flat, fn, out=self.hc_mix[:T], epi=ops.EPI_STORE_F32)
        ops.hc_split(self.hc, self.streams[:T], self.hc_mix[:T], base, scale, self.hc_coef[:T], x, T,
                     c.norm_eps, c.hc_eps, c.hc_sinkhorn_iters)
        tm.stop("hyper_connection")

    def _head(self, xs, n: int, norm_w, ids_out, logits_out=None):
        """Rows xs [n, d] (pre-norm) -> norm -> lm_head -> argmax ids (vocab-parallel)."""
        c, par = self.cfg, self.par
        xs = ops.rmsnorm(xs, norm_w, c.norm_eps, c.zero_centered_norm, out=self.x_last[:n])
        nv_head = isinstance(self.lm_head, ops.NvFp4Weight)
        if nv_head:
            ops.quantize_rows(xs, self.xq_head, n)
        if logits_out is not None:  # debug/numerics path: fp32 logits of this rank's vocab shard
            if nv_head:
                return ops.linear_nvfp4(self.xq_head, n, self.lm_head, out=logits_out[:n], epi=ops.EPI_STORE_F32)
            return ops.linear_bf16(xs, self.lm_head, out=logits_out[:n], epi=ops.EPI_STORE_F32)
        keys = self.keys[:n]
        n_valid = min(self.V_l, c.vocab_size - self.v_lo)
        if nv_head:
            w = self.lm_head
            ops.ext().gemm(w.packed, self.xq_head.packed, keys, ops.EPI_ARGMAX, w.n, w.k, n, ops._bn_for(n),
                           w.sf, self.xq_head.sf, w.gscale, self.xq_head.row_scale, None, None, None, None, None,
                           None, 0, 1, n_valid, ops.err_flag(self.dev), self.v_lo, 1, None, None)
        else:
            ops.lm_head_keys(xs, self.lm_head, keys, n_valid, self.v_lo)
        if par.tp > 1:
            # keys are u64 (orderable value << 32 | ~global id); flip the sign bit for a signed MAX
            keys.bitwise_xor_(-(1 << 63))
            par.all_reduce_max(keys)
            keys.bitwise_xor_(-(1 << 63))
        ops.argmax_finalize(keys, ids_out)
        return ids_out

    # ------------------------------------------------------------------ speculative decoding
    def capture_tap(self, i, x, T):
        """Keep the residual stream after layer i when the draft head taps it."""
        k = self.tap_slot.get(i) if getattr(self, "tap_slot", None) else None
        if k is not None:
            d = self.cfg.d_model
            self.taps[:T, k * d:(k + 1) * d].copy_(x[:T])

    def _mtp(self, h, ids, T, S, W_, decode, meta: Meta):
        """MTP block over T rows: h [T, d] target (or previous MTP) pre-norm hidden states,
        ids [T] the tokens that follow them.  Output (pre-norm) in self.x[:T]."""
        c, M, tm = self.cfg, self.mtp, self.timer
        tm.start("mtp")
        e = self.e_buf[:T]
        ops.embed(ids[:T], self.embed, e, 0)
        ops.rmsnorm(e, M.enorm, c.norm_eps, c.zero_centered_norm, out=e)
        hn = ops.rmsnorm(h, M.hnorm, c.norm_eps, c.zero_centered_norm, out=self.xn[:T])
        x = self.x[:T]
        ops.linear_bf16(hn, M.wh, out=x)  # hn is read before x is written (x may alias h)
        ops.linear_bf16(e, M.we, out=x, epi=ops.EPI_RESIDUAL_BF16, residual=x)
        self._block(M.layer, "mtp", x, T, S, W_, decode, meta)
        tm.stop("mtp")
        return x

    def spec_forward(self, T: int, S: int, W_: int, n_out: int, spec_rows: int, n_verify: int,
                     dummy_page: int, mtp_logits_out=None, draft_passes: int | None = None) -> torch.Tensor:
        """One speculative step (verify + accept + commit + K drafts), all on the device.

        Rows [0, spec_rows) are verify rows of the first n_verify sequences (each fed
        [last, d drafts], d <= K); the rest are prefill chunks.  Leaves in self.step_out:
        target ids of the sampled rows, accepted drafts per sequence, and the next drafts
        [K][S], of which the first `draft_passes` (default K) are produced this step.  With
        draft_passes 0 the MTP block still runs (its KV stays coherent) but no head does.
        """
        K = self.spec_k
        passes = K if draft_passes is None else draft_passes
        if not 0 <= passes <= K:
            raise ValueError(f"draft_passes {passes} outside 0..{K}")
        self.forward_replicated(T, S, W_, n_out, False, spec_rows=spec_rows)
        meta = self.main_meta()
        ops.ext().spec_accept(T, S, K, meta.ids, meta.q_start, meta.q_len, meta.pos, self.verify, self.sample,
                              self.out_ids, self.out_idx, self.next_tok, self.block_table, self.page_size,
                              dummy_page, self.n_acc, self.mtp_ids, self.mtp_rows, self.d_pos, self.d_slots,
                              self.d_kvlen)
        if n_verify and getattr(self, "dn_buf", None) is not None:
            b = self.dn_buf
            ops.ext().gdn_commit(b.state, b.conv_state, b.rk, b.rv, b.rg, b.rb, b.rx, meta.q_start, meta.state_slot,
                                 self.n_acc, n_verify, int(b.gate_ch))
        if self.mtp is None:
            if mtp_logits_out is not None:
                raise ValueError("the model has no MTP head")
            return self.step_out  # host-drafted speculation: verify + accept + commit only
        # draft pass 1: every row of the step (writes the MTP KV of all new positions); a
        # hidden-tap drafter reads the merged taps instead of the last layer's state
        h1 = self.x[:T]
        if self.mtp.wtap is not None:
            h1 = ops.linear_bf16(self.taps[:T], self.mtp.wtap, out=self.tap_h[:T])
        x = self._mtp(h1, self.mtp_ids, T, S, W_, False, meta)
        if passes == 0 and mtp_logits_out is None:
            return self.step_out
        hd = torch.index_select(x, 0, self.mtp_rows[:S], out=self.h_d[:S])
        if mtp_logits_out is not None:
            return self._head(hd, S, self.mtp.norm, None, logits_out=mtp_logits_out)
        self._head(hd, S, self.mtp.norm, self.drafts[0])
        # draft passes 2..passes: one row per sequence, chained on the previous MTP output
        self.d_nwork.fill_(S)
        h = hd
        for j in range(1, passes):
            dm = Meta(self.drafts[j - 1], self.d_pos[j - 1], self.d_slots[j - 1], self.d_arange, self.d_ones,
                      self.d_kvlen[j - 1], self.d_arange, self.d_zeros, self.d_nwork, self.d_zeros)
            x = self._mtp(h, self.drafts[j - 1], S, S, S, True, dm)
            h = x
            self._head(x, S, self.mtp.norm, self.drafts[j])
        return self.step_out

    def _attention(self, i, L, xn, x, T, W_, decode, lead, meta: Meta, post_norm=None):
        if L.mla is not None:
            self._mla(i, L, xn, x, T, lead, meta)
            return
        c = self.cfg
        D = c.head_dim
        tm = self.timer
        tm.start("attn.qkv")
        qkv = self._linear(xn, L.wqkv, self.qkv[:T], T=T, xq=self.xq_attn)
        if self.act_tap is not None and isinstance(L.wqkv, ops.NvFp4Weight):
            self.act_tap(i, "attn_in", self.xq_attn, T, None)
        if L.qkv_bias is not None:
            qkv[:, :L.qkv_bias.numel()].add_(L.qkv_bias)
        tm.stop("attn.qkv")
        li = self.attn_index[i]
        tm.start("attn.rope_kv")
        ops.qk_rope_kv(qkv, T, self.Hq, self.Hkv, D, c.rotary_dim, c.attn_output_gate, meta.pos[:T], self.inv_freq,
                       self.q[:T], self.gate[:T] if self.gate is not None else None, L.q_norm, L.k_norm, c.norm_eps,
                       c.zero_centered_norm, self.k_cache[li], self.v_cache[li], meta.slots[:T], self.page_size,
                       self.k_scales[li], self.v_scales[li])
        tm.stop("attn.rope_kv")
        if L.idx is not None:
            self._dsa(L, li, xn, T, meta)
        else:
            self._dense_attention(li, T, W_, decode, meta)
        tm.start("attn.o")
        if lead:
            self._linear(self.attn_out[:T], L.wo, x, epi=ops.EPI_RESIDUAL_BF16, residual=x, T=T,
                         xq=self.xq_attn_o, fused=self._norm_into_xn(post_norm, T) if post_norm is not None else None)
        else:
            self._linear(self.attn_out[:T], L.wo, x, T=T, xq=self.xq_attn_o)
        if self.act_tap is not None and isinstance(L.wo, ops.NvFp4Weight):
            self.act_tap(i, "attn_out", self.xq_attn_o, T, None)
        tm.stop("attn.o")

    def _mla(self, i, L, xn, x, T, lead, meta: Meta):
        """Absorbed NoPE MLA: low-rank query, latent write, (DSA selection), absorbed
        attention over the latent, value expansion, o_proj."""
        c, tm = self.cfg, self.timer
        ml = c.mla
        w_qa, qa_n, w_qb, w_kva, kva_n, wk, wv_t = L.mla
        li = self.attn_index[i]
        latent = self.k_cache[li].view(-1, ml.kv_lora_rank)
        tm.start("attn.qkv")
        ops.linear_bf16(xn, w_qa, out=self.q_lat[:T])
        ops.rmsnorm(self.q_lat[:T], qa_n, c.norm_eps, False, out=self.q_lat_n[:T])
        ops.linear_bf16(self.q_lat_n[:T], w_qb, out=self.q_nope[:T])
        ops.linear_bf16(xn, w_kva, out=self.kv_lat[:T])
        ops.ext().mla_latent_write(self.kv_lat[:T], kva_n, c.norm_eps, latent, meta.slots[:T], T)
        tm.stop("attn.qkv")
        sel = nsel = None
        if L.idx is not None:
            sa = c.sparse_attention
            w, knw, knb, ape = L.idx
            tm.start("attn.indexer")
            ops.linear_bf16(xn, w, out=self.idx_proj[:T])
            args = (self.idx_proj[:T], sa.index_heads, sa.index_dim, sa.kpool, sa.top_k, knw, knb, ape,
                    self.ik_cache[li], self.ig_cache[li], meta.slots[:T], meta.pos[:T], meta.q_start,
                    int(self._n_seqs), self.block_table, self.page_size)
            ops.ext().dsa_index_kv(*args, T)
            ops.ext().dsa_select(*args, self.dsa_scores[:T], self.dsa_sel[:T], self.dsa_nsel[:T], T)
            tm.stop("attn.indexer")
            sel, nsel = self.dsa_sel, self.dsa_nsel
        tm.start("attn.core")
        R = self.mla_rows
        for r0 in range(0, T, R):
            n = min(R, T - r0)
            ops.ext().mla_attention(self.q_nope[r0:r0 + n], wk, wv_t, latent, self.mla_qabs, self.mla_ctx,
                                    self.attn_out[r0:r0 + n], self.Hq, ml.qk_nope_head_dim, ml.v_head_dim,
                                    1.0 / math.sqrt(ml.qk_nope_head_dim), meta.pos[r0:r0 + n], meta.q_start,
                                    int(self._n_seqs), self.block_table, self.page_size,
                                    sel[r0:r0 + n] if sel is not None else None,
                                    nsel[r0:r0 + n] if nsel is not None else None, n, r0)
        tm.stop("attn.core")
        tm.start("attn.o")
        if lead:
            ops.linear_bf16(self.attn_out[:T], L.wo, out=x, epi=ops.EPI_RESIDUAL_BF16, residual=x)
        else:
            ops.linear_bf16(self.attn_out[:T], L.wo, out=x)
        tm.stop("attn.o")

    def _dsa(self, L, li, xn, T, meta: Meta):
        """Sparse attention: indexer GEMM, index-cache write, pool scores + top-k selection,
        GQA attention over the selected tokens."""
        c, tm = self.cfg, self.timer
        sa = c.sparse_attention
        w, knw, knb, ape = L.idx
        tm.start("attn.indexer")
        ops.linear_bf16(xn, w, out=self.idx_proj[:T])
        args = (self.idx_proj[:T], sa.index_heads, sa.index_dim, sa.kpool, sa.top_k, knw, knb, ape,
                self.ik_cache[li], self.ig_cache[li], meta.slots[:T], meta.pos[:T], meta.q_start,
                int(self._n_seqs), self.block_table, self.page_size)
        ops.ext().dsa_index_kv(*args, T)
        tm.stop("attn.indexer")
        tm.start("attn.core")
        D = c.head_dim
        ops.ext().dsa_attention(*args, self.dsa_scores[:T], self.dsa_sel[:T], self.dsa_nsel[:T], self.q[:T],
                                self.k_cache[li], self.v_cache[li], self.gate[:T] if self.gate is not None else None,
                                self.attn_out[:T].view(T, self.Hq, D), self.Hq, self.Hkv, D, 1.0 / math.sqrt(D), T)
        tm.stop("attn.core")

    def _dense_attention(self, li, T, W_, decode, meta: Meta):
        c, tm = self.cfg, self.timer
        D = c.head_dim
        splits = self.splits if decode else (self.vsplits if T <= self.max_out else 1)
        tm.start("attn.core")
        ops.attention(self.q[:T], self.attn_out[:T].view(T, self.Hq, D), self.k_cache[li], self.v_cache[li], self.Hq,
                      self.Hkv, D, self.block_table, meta.q_start, meta.q_len, meta.kv_len, meta.w_seq, meta.w_tok0,
                      meta.num_work, W_, gate=self.gate[:T] if self.gate is not None else None, num_splits=splits,
                      ws_o=self.ws_o if splits > 1 else None, ws_ml=self.ws_ml if splits > 1 else None,
                      page_size=self.page_size, decode=decode, k_scale=self.k_scales[li], v_scale=self.v_scales[li])
        tm.stop("attn.core")

    def _moe(self, L, xn, x, T, decode, lead, next_norm=None):
        """MoE sub-layer; returns True when its combine also wrote the next block's attention
        norm into xn (`next_norm`: resident experts, residual rank only)."""
        c = self.cfg
        # 32-token tiles while experts see few rows (decode, verify, short chunks); 128 otherwise
        few = T * self.k_out <= 32 * self.e_tot
        plan = self.plan_dec if (T <= self.plan_dec_tokens and (decode or few)) else self.plan_pre
        tm = self.timer
        tm.start("moe.router")
        logits = ops.linear_bf16(xn, L.router_w, out=self.logits[:T], epi=ops.EPI_STORE_F32)
        streamed = self.streamer is not None and id(L) in self.streamer.layers
        route = ops.router_topk if streamed else ops.route_and_plan  # streamed passes plan per pass
        route(logits, c.num_experts, c.top_k, c.num_shared_experts, c.router == "sigmoid",
              c.norm_topk_prob, c.routed_scaling, L.router_b,
              c.num_experts if c.shared_expert_gate else -1, plan, T,
              e_lo=self.e_lo, e_hi=self.e_lo + self.E_l, shared_local=self.shared_local)
        if self.telemetry is not None:
            # local expert index -> global id (the shared experts follow the local ones)
            ids = plan.ids[:T]
            order = torch.tensor(self.expert_order + [-1], dtype=torch.long, device=ids.device)
            ids = torch.where((ids >= 0) & (ids < self.E_l), ids + self.e_lo, torch.full_like(ids, -1))
            ids = order[ids.long()]  # router index -> expert id (-1 stays -1 via the sentinel)
            self.telemetry.router(self._cur_layer, logits[:T], c.num_experts, c.router == "sigmoid", ids)
        if streamed:
            # routed experts stream from the host: one pass per group of slot-resident experts
            ids0 = plan.ids[:T].clone()
            tm.stop("moe.router")
            for i, ids in enumerate(self.streamer.passes(L, ids0)):
                plan.ids[:T].copy_(ids)
                # the router counted original local ids; segment sizes must follow slot ids
                ops.moe_recount(plan, T)
                self._moe_experts(L, xn, x, T, plan, lead or i > 0, planned=False)
            plan.ids[:T].copy_(ids0)
            return False
        tm.stop("moe.router")
        return self._moe_experts(L, xn, x, T, plan, lead, planned=True, next_norm=next_norm)

    def _moe_experts(self, L, xn, x, T, plan, lead, planned=False, next_norm=None):
        """(Plan,) dispatch, both grouped GEMMs and the combine of one routing (x += the
        weighted expert outputs when `lead`, else x = them); with `next_norm` (and `lead`)
        the combine also writes RMSNorm(x) * next_norm into xn and this returns True."""
        tm = self.timer
        if not planned:
            tm.start("moe.router")  # the plan belongs to routing
            ops.moe_plan(plan)
            tm.stop("moe.router")
        tm.start("moe.dispatch")
        ops.moe_dispatch_quantize(xn, T, plan, self.xq)
        tm.stop("moe.dispatch")
        if self.act_tap is not None:
            self.act_tap(self._cur_layer, "moe_in", self.xq, T, plan)
        if self.sentinel:
            self.h.fill_(float("nan"))
            self.y.fill_(float("nan"))
        tm.start("moe.gemm1")
        ops.grouped_nvfp4(self.xq, L.w13, self.h, ops.EPI_SWIGLU, plan, plan.bn)
        tm.stop("moe.gemm1")
        tm.start("moe.quant_h")
        ops.quantize_assigned(self.h, T, plan, self.hq)
        tm.stop("moe.quant_h")
        if self.act_tap is not None:
            self.act_tap(self._cur_layer, "moe_h", self.hq, T, plan)
        tm.start("moe.gemm2")
        ops.grouped_nvfp4(self.hq, L.w2, self.y, ops.EPI_STORE_BF16, plan, plan.bn)
        tm.stop("moe.gemm2")
        if self.sentinel:
            self._check_sentinel(plan, T)
        tm.start("moe.combine")
        c = self.cfg
        norm = (next_norm, self.xn[:T], c.norm_eps, c.zero_centered_norm) if (next_norm is not None and lead) else None
        ops.moe_combine(self.y, plan, T, x if lead else None, x, norm=norm)
        tm.stop("moe.combine")
        return norm is not None

    def _check_sentinel(self, plan, T):
        """Every routed (token, k) row of both expert GEMM outputs was written."""
        k = plan.k_out
        rows = plan.pos[:T * k].view(T, k)[plan.ids[:T] >= 0].long()
        for name, buf in (("gemm1", self.h), ("gemm2", self.y)):
            bad = torch.isnan(buf[rows]).any(-1)
            if bool(bad.any()):
                raise RuntimeError(f"sentinel: MoE {name} of layer {self._cur_layer} left "
                                   f"{int(bad.sum())} of {rows.numel()} routed rows unwritten")

    def _dense(self, L, xn, x, T, lead, next_norm=None):
        """Dense SwiGLU MLP; returns True when the down projection also wrote the next
        block's attention norm into xn (`next_norm`, residual rank only)."""
        ops.quantize_rows(xn, self.xq_d, T)
        ops.linear_nvfp4(self.xq_d, T, L.w13, out=self.hd[:T], epi=ops.EPI_SWIGLU)
        ops.quantize_rows(self.hd[:T], self.hq_d, T)
        if self.act_tap is not None:
            self.act_tap(self._cur_layer, "dense_in", self.xq_d, T, None)
            self.act_tap(self._cur_layer, "dense_h", self.hq_d, T, None)
        if lead:
            f = self._norm_into_xn(next_norm, T) if next_norm is not None else None
            ops.linear_nvfp4(self.hq_d, T, L.w2, out=x, epi=ops.EPI_RESIDUAL_BF16, residual=x, fused=f)
            return f is not None
        ops.linear_nvfp4(self.hq_d, T, L.w2, out=x)
        return False
