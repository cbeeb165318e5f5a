"""Kernel microbenchmarks with roofline fractions.

    python -m rocket_b200.kbench --case moe_decode [--iters 10]

Each case builds inputs larger than L2 (126 MB) where the kernel is bandwidth
bound, runs warm-up launches, then times `iters` launches with CUDA events on
the launching stream (synchronize on both sides, an L2 flush between timed
launches) and prints one JSON line: achieved GB/s or TFLOP/s and the fraction
of the measured peaks in MEASURED_PEAKS.json (copy bandwidth / cuBLAS bf16).

Counterpart of the reference's microbenchmarks (engines/glm5-moe-nvfp4-2b/bench/
nvfp4_grouped_gemm.cu, kda_decode_step.cu, sparse_mla_decode.cu, ...).
"""
from __future__ import annotations

import argparse
import json
import math
import os

import torch

from . import ops

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


class Timer:
    def __init__(self):
        self.flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    def run(self, fn, warmup=3, iters=10):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        tot = 0.0
        for _ in range(iters):
            self.flush.zero_()  # evict L2 (256 MB > 126 MB)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            tot += a.elapsed_time(b)
        return tot / iters


def _random_nvfp4(n, k, experts, dev, fuse=False):
    from .models.weights import random_nvfp4_on_device
    g = torch.Generator(device=dev).manual_seed(0)
    return random_nvfp4_on_device((n, k), experts, 0.02, g, dev, fuse_swiglu=fuse)


def case_moe(tokens: int, experts=160, topk=8, d=5120, inter=1536, which="w13", bn=None):
    dev = torch.device("cuda")
    E_tot = experts + 1
    if which == "w13":
        w = _random_nvfp4(2 * inter, d, E_tot, dev, fuse=True)
        k = d
    else:
        w = _random_nvfp4(d, inter, E_tot, dev)
        k = inter
    if bn is None:
        bn = 32 if tokens * (topk + 1) / E_tot <= 32 else 128
    plan = ops.MoePlan(tokens, topk + 1, E_tot, bn, dev)
    logits = torch.randn(tokens, experts, device=dev)
    ops.router_topk(logits, experts, topk, 1, True, True, 1.0, None, -1, plan, tokens)
    ops.moe_plan(plan)
    x = torch.randn(tokens, k, device=dev).bfloat16()
    xq = ops.NvFp4Act(plan.max_rows, k, dev)
    ops.moe_dispatch_quantize(x, tokens, plan, xq)
    out = torch.empty(plan.max_rows, w.n // 2 if which == "w13" else w.n, dtype=torch.bfloat16, device=dev)
    epi = ops.EPI_SWIGLU if which == "w13" else ops.EPI_STORE_BF16
    fn = lambda: ops.grouped_nvfp4(xq, w, out, epi, plan, bn)
    nb = int(plan.num_blocks.item())
    ids = plan.ids[:tokens].cpu()
    touched = len(set(ids.flatten().tolist()))
    wbytes = touched * (w.packed.numel() + w.sf.numel()) / E_tot
    flops = 2.0 * tokens * (topk + 1) * w.n * k
    return fn, {"bytes": wbytes, "flops": flops, "touched_experts": touched, "blocks": nb, "bn": bn}


def case_linear_bf16(m, n, k, splits=None):
    dev = torch.device("cuda")
    x = torch.randn(m, k, device=dev).bfloat16()
    w = (torch.randn(n, k, device=dev) * 0.02).bfloat16()
    out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    fn = lambda: ops.linear_bf16(x, w, out=out, splits=splits)
    return fn, {"bytes": n * k * 2 + m * k * 2 + m * n * 2, "flops": 2.0 * m * n * k,
                "splits": ops.pick_splits(m, n, k, False) if splits is None else splits}


def case_linear_fp8(m, n, k):
    """FP8-row GEMM including the per-token activation quantizer (both timed)."""
    dev = torch.device("cuda")
    x = torch.randn(m, k, device=dev).bfloat16()
    w = ops.Fp8Weight.quantize(torch.randn(n, k, device=dev) * 0.02)
    xq = ops.Fp8Act(m, k, dev)
    out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)

    def fn():
        ops.quantize_rows_fp8(x, xq, m)
        ops.linear_fp8(xq, m, w, out=out)
    return fn, {"bytes": n * k + n * 4 + m * k * 3 + m * n * 2, "flops": 2.0 * m * n * k,
                "splits": ops.pick_splits(m, n, k // 2, False)}


def case_dsa_decode(S=64, ctx=8192, top_k=2048):
    """DSA indexer scores + top-k selection + sparse GQA attention for one decode row per
    sequence at context `ctx` (96 q / 8 kv heads x 128, 32 indexer heads, pools of 4)."""
    dev = torch.device("cuda")
    Hq, Hkv, D, Hi, Di, kp = 96, 8, 128, 32, 128, 4
    kc, vc, bt = _paged_kv(S, Hkv, D, ctx, dev)
    n_slots = kc.shape[0] * 64
    ik = torch.randn(n_slots, Di, device=dev).bfloat16()
    ig = torch.randn(n_slots, Di, device=dev).bfloat16()
    cols = Hi * Di + 2 * Di + Hi
    proj = torch.randn(S, (cols + 127) // 128 * 128, device=dev).bfloat16()
    i32 = lambda v: torch.tensor(v, dtype=torch.int32, device=dev)
    pos = i32([ctx - 1] * S)
    qs = i32(list(range(S)))
    slots = i32([int(bt[s, (ctx - 1) // 64]) * 64 + (ctx - 1) % 64 for s in range(S)])
    knw, knb = torch.ones(Di, device=dev), torch.zeros(Di, device=dev)
    ape = torch.randn(kp, Di, device=dev)
    scores = torch.zeros(S, ctx // kp, device=dev)
    sel = torch.zeros(S, top_k + kp - 1, dtype=torch.int32, device=dev)
    nsel = torch.zeros(S, dtype=torch.int32, device=dev)
    q = torch.randn(S, Hq, D, device=dev).bfloat16()
    out = torch.empty(S, Hq, D, dtype=torch.bfloat16, device=dev)
    args = (proj, Hi, Di, kp, top_k, knw, knb, ape, ik, ig, slots, pos, qs, S, bt, 64)
    fn = lambda: ops.ext().dsa_attention(*args, scores, sel, nsel, q, kc, vc, None, out, Hq, Hkv, D,
                                         1.0 / math.sqrt(D), S)
    idx_bytes = S * ctx * Di * 2 * 2          # keys + gates of every visible token
    kv_bytes = S * min(ctx, top_k) * Hkv * D * 2 * 2
    return fn, {"bytes": idx_bytes + kv_bytes, "flops": 2.0 * S * (ctx // kp) * Hi * Di}


def _paged_kv(S, Hkv, D, ctx, dev, page=64, kv="bf16"):
    pages_per = -(-ctx // page)
    num_pages = S * pages_per + 1
    kd = torch.float8_e4m3fn if kv == "fp8" else torch.bfloat16
    kc = torch.randn(num_pages, Hkv, page, D, device=dev).to(kd)
    vc = torch.randn(num_pages, Hkv, D, page, device=dev).to(kd)
    bt = torch.arange(S * pages_per, dtype=torch.int32, device=dev).view(S, pages_per)
    return kc, vc, bt


def case_attn_decode(S=64, Hq=96, Hkv=8, D=128, ctx=2048, splits=None, kv="bf16"):
    dev = torch.device("cuda")
    kc, vc, bt = _paged_kv(S, Hkv, D, ctx, dev, kv=kv)
    q = torch.randn(S, Hq, D, device=dev).bfloat16()
    out = torch.empty_like(q)
    i32 = lambda a: torch.tensor(a, dtype=torch.int32, device=dev)
    if splits is None:
        items, best, best_e = S * Hkv, 1, 0
        for s in range(1, 9):
            e = items * s / (math.ceil(items * s / ops.num_sms()) * ops.num_sms())
            if e > best_e + 0.01:
                best, best_e = s, e
        splits = best
    ws_o = torch.empty(splits, S * Hq, D, device=dev) if splits > 1 else None
    ws_ml = torch.empty(splits, S * Hq, 2, device=dev) if splits > 1 else None
    args = (q, out, kc, vc, Hq, Hkv, D, bt, i32(list(range(S))), i32([1] * S), i32([ctx] * S), i32(list(range(S))),
            i32([0] * S), i32([S]), S)
    fn = lambda: ops.attention(*args, num_splits=splits, ws_o=ws_o, ws_ml=ws_ml, decode=True)
    nbytes = S * ctx * Hkv * D * 2 * (1 if kv == "fp8" else 2)
    return fn, {"bytes": nbytes, "flops": 4.0 * S * Hq * ctx * D, "splits": splits, "kv": kv}


def case_attn_prefill(S=4, Hq=96, Hkv=8, D=128, L=2048, kv="bf16", block_n=0):
    dev = torch.device("cuda")
    kc, vc, bt = _paged_kv(S, Hkv, D, L, dev, kv=kv)
    T = S * L
    q = torch.randn(T, Hq, D, device=dev).bfloat16()
    out = torch.empty_like(q)
    i32 = lambda a: torch.tensor(a, dtype=torch.int32, device=dev)
    w_seq, w_tok0 = ops.attention_work([L] * S, Hq, Hkv)
    args = (q, out, kc, vc, Hq, Hkv, D, bt, i32([s * L for s in range(S)]), i32([L] * S), i32([L] * S),
            i32(w_seq), i32(w_tok0), i32([len(w_seq)]), len(w_seq))
    fn = lambda: ops.attention(*args, block_n=block_n)
    return fn, {"bytes": S * L * Hkv * D * 4 + T * Hq * D * 4, "flops": 4.0 * S * Hq * D * L * L / 2,
                "block_n": block_n or 64}


def case_gdn_decode(S=32, Hk=16, Hv=32, D=128, K=4, kda=False, one_token=1):
    """One gated-DeltaNet layer decode step (Qwen3-Next shape): conv+prep, recurrent
    scan over the fp32 state of every sequence, conv-state shift.  `kda`: per-channel
    (Kimi delta attention) decay gates.  `one_token` 0: the scan and gated-norm launches
    instead of the fused one-token kernel."""
    dev = torch.device("cuda")
    C = 2 * Hk * D + Hv * D
    rows = C + Hv * D + 2 * Hv
    f32 = dict(dtype=torch.float32, device=dev)
    i32 = lambda a: torch.tensor(a, dtype=torch.int32, device=dev)
    proj = torch.randn(S, rows, device=dev).bfloat16()
    conv_w = (torch.randn(C, K, device=dev) * 0.5).bfloat16()
    conv_state = torch.randn(S + 1, K - 1, C, device=dev).bfloat16()
    state = torch.randn(S + 1, Hv, D, D, **f32) * 0.01
    q, k = torch.zeros(S, Hk, D, **f32), torch.zeros(S, Hk, D, **f32)
    v = torch.zeros(S, Hv, D, **f32)
    beta, g = torch.zeros(S, Hv, **f32), torch.zeros(S, Hv * (D if kda else 1), **f32)
    out = torch.zeros(S, Hv * D, dtype=torch.bfloat16, device=dev)
    o_raw = torch.zeros(S, Hv, D, **f32)
    A_log, dt_bias = torch.zeros(Hv, **f32), torch.ones(Hv, **f32)
    norm_w = torch.ones(D, dtype=torch.bfloat16, device=dev)
    pos, qs, ql, slot = i32([100] * S), i32(list(range(S))), i32([1] * S), i32(list(range(S)))
    fn = lambda: ops.ext().gdn(proj, conv_w, conv_state, A_log, dt_bias, norm_w, q, k, v, beta, g, state, out, pos,
                               qs, ql, slot, Hk, Hv, K, C, 1e-6, S, S, 0, None, None, None, None, None, int(kda), -5.0,
                               int(kda), o_raw, one_token)
    nbytes = 2 * S * Hv * D * D * 4 + S * rows * 2 + 2 * S * (K - 1) * C * 2 + S * Hv * D * 2
    return fn, {"bytes": nbytes, "flops": 6.0 * S * Hv * D * D}


def case_gdn_prefill(T=2048, Hk=16, Hv=32, D=128, K=4):
    """One gated-DeltaNet layer over a T-token prompt chunk of one sequence (Qwen3-Next
    shape): the scan is sequential in the tokens, so this measures the per-token chain."""
    dev = torch.device("cuda")
    C = 2 * Hk * D + Hv * D
    rows = C + Hv * D + 2 * Hv
    f32 = dict(dtype=torch.float32, device=dev)
    i32 = lambda a: torch.tensor(a, dtype=torch.int32, device=dev)
    proj = (torch.randn(T, rows, device=dev) * 0.5).bfloat16()
    conv_w = (torch.randn(C, K, device=dev) * 0.5).bfloat16()
    conv_state = torch.zeros(2, K - 1, C, device=dev).bfloat16()
    state = torch.zeros(2, Hv, D, D, **f32)
    q, k = torch.zeros(T, Hk, D, **f32), torch.zeros(T, Hk, D, **f32)
    v = torch.zeros(T, Hv, D, **f32)
    beta, g = torch.zeros(T, Hv, **f32), torch.zeros(T, Hv, **f32)
    out = torch.zeros(T, Hv * D, dtype=torch.bfloat16, device=dev)
    o_raw = torch.zeros(T, Hv, D, **f32)
    A_log, dt_bias = torch.zeros(Hv, **f32), torch.ones(Hv, **f32)
    norm_w = torch.ones(D, dtype=torch.bfloat16, device=dev)
    pos, qs, ql, slot = i32(list(range(T))), i32([0]), i32([T]), i32([0])
    fn = lambda: ops.ext().gdn(proj, conv_w, conv_state, A_log, dt_bias, norm_w, q, k, v, beta, g, state, out, pos,
                               qs, ql, slot, Hk, Hv, K, C, 1e-6, T, 1, 0, None, None, None, None, None, 0, -5.0, 0,
                               o_raw, 1)
    return fn, {"bytes": T * rows * 2 + 2 * Hv * D * D * 4 + T * Hv * D * 2, "flops": 6.0 * T * Hv * D * D}


def case_rmsnorm(T=8192, d=5120):
    dev = torch.device("cuda")
    x = torch.randn(T, d, device=dev).bfloat16()
    w = torch.ones(d, dtype=torch.bfloat16, device=dev)
    out = torch.empty_like(x)
    return (lambda: ops.rmsnorm(x, w, 1e-6, False, out=out)), {"bytes": 2 * T * d * 2, "flops": 4.0 * T * d}


def case_rope_kv(T=8192, Hq=96, Hkv=8, D=128):
    dev = torch.device("cuda")
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device=dev).bfloat16()
    pos = torch.arange(T, dtype=torch.int32, device=dev)
    inv = ops.rope_inv_freq(D, 1e6, dev)
    q_out = torch.empty(T, Hq, D, dtype=torch.bfloat16, device=dev)
    pages = T // 64 + 1
    kc = torch.zeros(pages, Hkv, 64, D, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros(pages, Hkv, D, 64, dtype=torch.bfloat16, device=dev)
    fn = lambda: ops.qk_rope_kv(qkv, T, Hq, Hkv, D, D, False, pos, inv, q_out, k_cache=kc, v_cache=vc,
                                slot_mapping=pos, page_size=64)
    return fn, {"bytes": 2 * T * (Hq + 2 * Hkv) * D * 2, "flops": 6.0 * T * (Hq + Hkv) * D}


def case_router_quant(tokens=4096, experts=160, topk=8, d=5120):
    """Router top-k + plan + NVFP4 dispatch quantize of one prefill chunk."""
    dev = torch.device("cuda")
    E_tot = experts + 1
    plan = ops.MoePlan(tokens, topk + 1, E_tot, 128, dev)
    logits = torch.randn(tokens, experts, device=dev)
    x = torch.randn(tokens, d, device=dev).bfloat16()
    xq = ops.NvFp4Act(plan.max_rows, d, dev)

    def fn():
        ops.router_topk(logits, experts, topk, 1, True, True, 1.0, None, -1, plan, tokens)
        ops.moe_plan(plan)
        ops.moe_dispatch_quantize(x, tokens, plan, xq)
    rows = tokens * (topk + 1)
    return fn, {"bytes": tokens * d * 2 + rows * (d // 2 + d // 16), "flops": 0.0}


def case_router(tokens=64, experts=160, topk=8):
    """Sigmoid + bias router top-k (GLM-style, normalised, scaled) of `tokens` rows."""
    dev = torch.device("cuda")
    plan = ops.MoePlan(tokens, topk, experts, 128, dev)
    logits = torch.randn(tokens, experts, device=dev)
    bias = torch.randn(experts, device=dev) * 0.1

    fn = lambda: ops.router_topk(logits, experts, topk, 0, True, True, 2.5, bias, -1, plan, tokens)
    return fn, {"bytes": tokens * experts * 4 + tokens * topk * 8, "flops": 0.0}


def case_router_plan(tokens=64, experts=160, topk=8, shared=1, bn=32):
    """Router top-k and MoE plan in one launch (the model's decode path): GLM-style sigmoid +
    bias routing with a shared expert, block list for token tile `bn`."""
    dev = torch.device("cuda")
    plan = ops.MoePlan(tokens, topk + shared, experts + shared, bn, dev)
    logits = torch.randn(tokens, experts, device=dev)
    bias = torch.randn(experts, device=dev) * 0.1

    fn = lambda: ops.route_and_plan(logits, experts, topk, shared, True, True, 2.5, bias, -1, plan, tokens)
    return fn, {"bytes": tokens * experts * 4 + tokens * (topk + shared) * 8, "flops": 0.0}


def case_nvfp4_quant(rows=4096, k=5120):
    """NVFP4 quantization of bf16 activation rows (e2m1 + e4m3 block scales)."""
    dev = torch.device("cuda")
    x = torch.randn(rows, k, device=dev).bfloat16()
    out = ops.NvFp4Act(rows, k, dev)
    return (lambda: ops.quantize_rows(x, out, rows)), {"bytes": rows * k * 2 + rows * (k // 2 + k // 16),
                                                       "flops": 0.0}


# ----------------------------------------------------------------- reference controls
# The same workloads on the reference's own SIMT kernels (rocket_b200/refcontrols.py builds
# them unchanged into baseline/_ref/controls.so): `--impl reference`.
def _ref_lib():
    from . import refcontrols
    lib = refcontrols.load()
    if lib is None:
        raise RuntimeError("reference controls not built (python -m rocket_b200.refcontrols build)")
    return lib


def ref_rmsnorm(T=8192, d=5120):
    lib, dev = _ref_lib(), torch.device("cuda")
    x = torch.randn(T, d, device=dev).bfloat16()
    w = torch.ones(d, dtype=torch.bfloat16, device=dev)
    out = torch.empty_like(x)
    st = lambda: torch.cuda.current_stream().cuda_stream
    fn = lambda: lib.ctl_rmsnorm(out.data_ptr(), x.data_ptr(), w.data_ptr(), T, d, 1e-6, st())
    return fn, {"bytes": 2 * T * d * 2, "flops": 4.0 * T * d}


def ref_router(tokens=64, experts=160, topk=8):
    lib, dev = _ref_lib(), torch.device("cuda")
    logits = torch.randn(tokens, experts, device=dev)
    bias = torch.randn(experts, device=dev) * 0.1
    idx = torch.empty(tokens, topk, dtype=torch.int32, device=dev)
    w = torch.empty(tokens, topk, device=dev)
    st = lambda: torch.cuda.current_stream().cuda_stream
    fn = lambda: lib.ctl_moe_router(idx.data_ptr(), w.data_ptr(), logits.data_ptr(), bias.data_ptr(), tokens,
                                    experts, topk, 1, 2.5, st())
    return fn, {"bytes": tokens * experts * 4 + tokens * topk * 8, "flops": 0.0}


def ref_nvfp4_quant(rows=4096, k=5120):
    lib, dev = _ref_lib(), torch.device("cuda")
    x = torch.randn(rows, k, device=dev).bfloat16()
    packed = torch.empty(rows, k // 2, dtype=torch.uint8, device=dev)
    sf = torch.zeros((rows + 127) // 128 * 128 * (k // 16), dtype=torch.uint8, device=dev)
    row_in = torch.arange(rows, dtype=torch.int32, device=dev)
    grp = torch.zeros(rows, dtype=torch.int32, device=dev)
    base = torch.zeros(1, dtype=torch.int64, device=dev)
    st = lambda: torch.cuda.current_stream().cuda_stream
    fn = lambda: lib.ctl_nvfp4_quantize_rows(packed.data_ptr(), sf.data_ptr(), x.data_ptr(), row_in.data_ptr(),
                                             grp.data_ptr(), base.data_ptr(), rows, k, st())
    return fn, {"bytes": rows * k * 2 + rows * (k // 2 + k // 16), "flops": 0.0}


def ref_kda_step(S=32, H=64, D=128):
    """The reference's KDA decode step alone (its recurrent kernel: state read + write);
    the matching framework case `kda_decode_bs32` runs the whole layer step."""
    lib, dev = _ref_lib(), torch.device("cuda")
    state = torch.randn(S, H, D, D, device=dev) * 0.01
    q, k, v = (torch.randn(S, H * D, device=dev).bfloat16() * 0.1 for _ in range(3))
    g = -torch.rand(S, H * D, device=dev).bfloat16() * 0.1
    beta = torch.rand(S, H, device=dev).bfloat16()
    o = torch.empty(S, H * D, dtype=torch.bfloat16, device=dev)
    st = lambda: torch.cuda.current_stream().cuda_stream
    fn = lambda: lib.ctl_kda_step(state.data_ptr(), o.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                  g.data_ptr(), beta.data_ptr(), S, H, D, H * D, st())
    return fn, {"bytes": 2 * S * H * D * D * 4, "flops": 6.0 * S * H * D * D}


REF_CASES = {
    "rmsnorm_prefill": ref_rmsnorm,
    "router_decode": lambda: ref_router(64),
    "router_prefill": lambda: ref_router(4096),
    "nvfp4_quant_prefill": ref_nvfp4_quant,
    "kda_decode_bs32": ref_kda_step,
}


def case_small_chain(pdl: bool, n: int = 128, rows: int = 64, d: int = 5120):
    """A CUDA graph of `n` dependent decode-sized kernels (RMSNorm of 64 rows x 5120, each
    reading the previous output): launch-latency bound; with `pdl` every launch is
    programmatic (the next kernel is scheduled while this one drains)."""
    dev = torch.device("cuda")
    bufs = [torch.randn(rows, d, device=dev).bfloat16() for _ in range(2)]
    w = torch.ones(d, dtype=torch.bfloat16, device=dev)
    prev = ops.pdl_enabled()
    ops.set_pdl(pdl)
    try:
        def body():
            for i in range(n):
                ops.rmsnorm(bufs[i % 2], w, 1e-6, False, out=bufs[(i + 1) % 2])
        body()
        torch.cuda.synchronize()
        s = torch.cuda.Stream()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            body()
    finally:
        ops.set_pdl(prev)
    return g.replay, {"bytes": n * 2 * rows * d * 2, "flops": 0.0, "launches": n}


def case_expert_slot_fill(experts: int = 16, d: int = 5120, inter: int = 1536):
    """Host -> device copies of streamed experts into device slots (pinned source): the
    w13 + w2 NVFP4 bytes of `experts` GLM-shaped experts per launch group."""
    import types

    from .models.expert_stream import ExpertStreamer
    dev = torch.device("cuda")
    L = types.SimpleNamespace(w13=_random_nvfp4(2 * inter, d, 64, dev, fuse=True), w2=_random_nvfp4(d, inter, 64, dev),
                              moe=True)
    st = ExpertStreamer(64, 0, experts, dev)
    st.adopt(L)
    h13, h2, _ = st.layers[id(L)]
    per = h13.pk + h13.sf + 4 * h13.gs + h2.pk + h2.sf + 4 * h2.gs

    def fn():
        for e in range(experts):
            h13.load(L.w13, e, e)
            h2.load(L.w2, e, e)
    return fn, {"bytes": experts * per, "flops": 0.0}


CASES = {
    "small_chain": lambda: case_small_chain(False),
    "small_chain_pdl": lambda: case_small_chain(True),
    "expert_slot_fill": lambda: case_expert_slot_fill(),
    "moe_decode_w13": lambda: case_moe(64, which="w13"),
    "moe_decode_w2": lambda: case_moe(64, which="w2"),
    "moe_prefill_w13": lambda: case_moe(4096, which="w13"),
    "moe_prefill8k_w13": lambda: case_moe(8192, which="w13"),
    "moe_prefill8k_w13_bn256": lambda: case_moe(8192, which="w13", bn=256),
    "moe_prefill8k_w2": lambda: case_moe(8192, which="w2"),
    "moe_prefill8k_w2_bn256": lambda: case_moe(8192, which="w2", bn=256),
    "lm_head_decode": lambda: case_linear_bf16(64, 151552, 5120),
    "o_proj_decode": lambda: case_linear_bf16(64, 5120, 12288),
    "qkv_decode": lambda: case_linear_bf16(64, 14336, 5120),
    "qkv_prefill": lambda: case_linear_bf16(8192, 14336, 5120),
    "attn_decode": lambda: case_attn_decode(),
    "attn_prefill": lambda: case_attn_prefill(),
    "moe_hybrid_verify_w13": lambda: case_moe(128, experts=512, topk=10, d=2048, inter=512, which="w13"),
    "moe_hybrid_verify_w2": lambda: case_moe(128, experts=512, topk=10, d=2048, inter=512, which="w2"),
    "gdn_decode_bs32": lambda: case_gdn_decode(),
    "gdn_prefill_2k": lambda: case_gdn_prefill(),
    "rmsnorm_prefill": lambda: case_rmsnorm(),
    "rope_kv_prefill": lambda: case_rope_kv(),
    "rope_kv_decode": lambda: case_rope_kv(T=64),
    "router_quant_decode": lambda: case_router_quant(tokens=64),
    "router_quant_prefill": lambda: case_router_quant(),
    "attn_decode_fp8": lambda: case_attn_decode(kv="fp8"),
    "attn_decode_fp8_ctx16k": lambda: case_attn_decode(ctx=16384, kv="fp8"),
    "attn_decode_ctx16k": lambda: case_attn_decode(ctx=16384),
    "attn_prefill_fp8": lambda: case_attn_prefill(kv="fp8"),
    "attn_prefill_bn128": lambda: case_attn_prefill(block_n=128),
    "o_proj_decode_fp8": lambda: case_linear_fp8(64, 5120, 12288),
    "qkv_prefill_fp8": lambda: case_linear_fp8(8192, 14336, 5120),
    "dsa_decode_ctx8k": lambda: case_dsa_decode(),
    "router_decode": lambda: case_router(64),
    "router_prefill": lambda: case_router(4096),
    "router_plan_decode": lambda: case_router_plan(64),
    "router_plan_decode256": lambda: case_router_plan(256),
    "nvfp4_quant_prefill": lambda: case_nvfp4_quant(),
    "kda_decode_bs32": lambda: case_gdn_decode(S=32, Hk=64, Hv=64, kda=True),
}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default="all")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="rocket", choices=["rocket", "reference"],
                    help="reference: the same workloads on the reference's SIMT kernels (controls)")
    a = ap.parse_args(argv)
    pk = peaks()
    t = Timer()
    table = REF_CASES if a.impl == "reference" else CASES
    names = list(table) if a.case == "all" else a.case.split(",")
    for name in names:
        if name not in table:
            print(json.dumps({"case": name, "impl": a.impl, "skipped": "no such case for this impl"}), flush=True)
            continue
        try:
            fn, info = table[name]()
        except RuntimeError as e:  # a case this build cannot run (e.g. PDL without its build flag)
            print(json.dumps({"case": name, "skipped": str(e)}), flush=True)
            continue
        ms = t.run(fn, a.warmup, a.iters)
        ops.check_errors()
        gbs = info["bytes"] / (ms * 1e-3) / 1e9
        tfl = info["flops"] / (ms * 1e-3) / 1e12
        if "launches" in info:
            info["us_per_launch"] = round(ms * 1e3 / info["launches"], 3)
        print(json.dumps({"case": name, "impl": a.impl, "ms": round(ms, 4), "GB/s": round(gbs, 1),
                          "hbm_frac": round(gbs / pk["hbm_gbs"], 3), "TFLOP/s": round(tfl, 1),
                          "bf16_frac": round(tfl / pk["bf16_tflops"], 3), "peaks": pk["src"],
                          **{k: v for k, v in info.items() if k not in ("bytes", "flops")}}), flush=True)
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
