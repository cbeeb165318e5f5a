"""Expert-parallel NVFP4 MoE microbenchmark: fused P2P dispatch / combine vs NCCL.

    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \\
        -m rocket_b200.parallel.ep_bench [--tokens 4096 --hidden 4096 --experts 128 --top-k 8 --inter 1536]

Workload (the expert-parallel MoE microbenchmark): every GPU holds `tokens` bf16 activations ~N(0,1) of
width `hidden`; router logits come from a bf16 router GEMM, softmax top-k over
`experts` experts split evenly over the ranks (EP = world size); each expert is a
SwiGLU FFN (`inter`) with NVFP4 weights ~N(0,0.02).  One MoE block =
route -> dispatch -> gate/up GEMM -> SiLU*up -> down GEMM -> combine.

  fused  one process group of sm_100a kernels over CUDA-IPC peer memory:
         dispatch kernel (top-k + NVFP4 quantize + push of each routed row into its
         owner's per-(expert, source) slot), owner plan (waits for every source;
         blocks over the filled slots only), grouped GEMM1 with the SwiGLU epilogue,
         NVFP4 re-quantize, grouped GEMM2 whose epilogue pushes every output row back
         to its source, and a landing kernel that sums each token's k rows in fixed
         slot order (plus the residual).  No NCCL call on the path.
  nccl   the unfused baseline: torch top-k, sort rows by owner, NCCL all-to-all of
         the bf16 rows (variable splits), local grouped GEMMs (the same kernels),
         NCCL all-to-all back, weighted sum.

Timing: CUDA events on the launching stream, warm-up first, an L2 flush between
timed iterations, max over ranks.  The roofline of a path is the slower of the
tensor-core time (NVFP4 FLOPs at the dense FP4 peak scaled by the measured / nominal
bf16 ratio) and the bytes this GPU must push over NVLink at the measured 770 GB/s
per direction.  Counterpart of the reference's EP exchange and its
nvfp4_grouped_gemm microbenchmark (engines/glm5-moe-nvfp4-2b/src/fabric/
expert_parallel.h:51-130, bench/nvfp4_grouped_gemm.cu).
"""
from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

from .. import ops
from ..models.weights import random_nvfp4_on_device
from .symm import SymmetricHeap

NVLINK_GBS = 770.0           # measured peer copy per direction per GPU on this pool
FP4_NOMINAL_TFLOPS = 9000.0  # dense NVFP4 per GPU
BF16_NOMINAL_TFLOPS = 2250.0
DISP, COMB = 2, 3
LAND_COMB, OUT_LOCAL = 2, 0


class EpMoE:
    def __init__(self, par, T: int, d: int, E: int, top_k: int, inter: int, seed: int = 0, bn: int = 128):
        self.par, self.T, self.d, self.E, self.k, self.inter = par, T, d, E, top_k, inter
        self.bn = bn  # token tile of the fused path's grouped GEMMs (and its owner-plan blocks)
        N = par.world
        self.N = N
        if E % N:
            raise ValueError("experts must divide the world size")
        self.E_l = E // N
        dev = par.device
        self.dev = dev
        g = torch.Generator(device=dev)
        g.manual_seed(seed * 7919 + par.rank)
        g_rep = torch.Generator(device=dev)
        g_rep.manual_seed(seed * 7919 + 100003)
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.x = torch.randn(T, d, generator=g, **bf)
        self.E_pad = (E + 127) // 128 * 128
        self.router_w = torch.zeros(self.E_pad, d, **bf)
        self.router_w[:E] = torch.randn(E, d, generator=g_rep, **bf) * 0.02
        self.w13 = random_nvfp4_on_device((2 * inter, d), self.E_l, 0.02, g, dev, fuse_swiglu=True)
        self.w2 = random_nvfp4_on_device((d, inter), self.E_l, 0.02, g, dev)
        self.logits = torch.zeros(T, self.E_pad, dtype=torch.float32, device=dev)
        self.err = ops.err_flag(dev)
        # ---- fused path: symmetric heap regions (identical layout on every rank)
        self.cap = T                                   # rows one source can send to one expert
        self.seg_rows = N * self.cap                   # per-expert segment: [source][cap]
        self.moe_rows = self.E_l * self.seg_rows
        sizes = {"xq": self.moe_rows * d // 2, "xsf": self.moe_rows // 128 * (d // 64) * 512,
                 "xrs": self.moe_rows * 4, "meta": self.moe_rows * 4, "cnt": self.E_l * 8 * 4,
                 "comb": T * top_k * d * 2}
        self.heap = SymmetricHeap(par, sum(s + 1024 for s in sizes.values()), slot=0)
        self.off = {k: self.heap.alloc(v) for k, v in sizes.items()}
        H = self.heap
        i32 = dict(dtype=torch.int32, device=dev)
        self.xq = ops.NvFp4Act.__new__(ops.NvFp4Act)
        self.xq.packed = H.view(self.off["xq"], (self.moe_rows, d // 2), torch.uint8)
        self.xq.sf = H.view(self.off["xsf"], (sizes["xsf"],), torch.uint8)
        self.xq.row_scale = H.view(self.off["xrs"], (self.moe_rows,), torch.float32)
        self.xq.k, self.xq.rows = d, self.moe_rows
        self.meta = H.view(self.off["meta"], (self.moe_rows,), torch.int32)
        self.cnt = H.view(self.off["cnt"], (self.E_l, 8), torch.int32)
        self.comb = H.view(self.off["comb"], (T, top_k, d), torch.bfloat16)
        self.comb_w = torch.zeros(T, top_k, dtype=torch.float32, device=dev)
        self.cnt_local = torch.zeros(E, **i32)
        self.max_blocks = self.E_l * (self.seg_rows // 128)
        self.blk = [torch.zeros(self.max_blocks, **i32) for _ in range(3)] + [torch.zeros(1, **i32)]
        self.row_list = torch.zeros(self.moe_rows, **i32)
        self.num_rows = torch.zeros(1, **i32)
        self.h = torch.zeros(self.moe_rows, inter, **bf)
        self.hq = ops.NvFp4Act(self.moe_rows, inter, dev)
        self.xres = torch.zeros(T, d, **bf)
        self.xn = torch.zeros(T, d, **bf)
        self.norm_w = torch.ones(d, **bf)
        # ---- NCCL baseline buffers (received rows <= T * k * N in the worst case)
        rmax = T * top_k * N
        self.plan_l = ops.MoePlan(rmax, 1, self.E_l, 128, dev)
        self.xq_l = ops.NvFp4Act(self.plan_l.max_rows, d, dev)
        self.h_l = torch.zeros(self.plan_l.max_rows, inter, **bf)
        self.hq_l = ops.NvFp4Act(self.plan_l.max_rows, inter, dev)
        self.y_l = torch.zeros(self.plan_l.max_rows, d, **bf)
        self.stats = {}

    # ------------------------------------------------------------------ fused
    def fused(self) -> torch.Tensor:
        T, d = self.T, self.d
        slot = self.heap.slot
        ops.linear_bf16(self.x, self.router_w, out=self.logits, epi=ops.EPI_STORE_F32)
        self.xres.zero_()
        args = {
            "logits": self.logits, "ld_logits": self.E_pad, "E": self.E, "top_k": self.k, "n_shared": 0,
            "sigmoid": 0, "norm_topk": 0, "shared_gate_col": -1, "scaling": 1.0, "bias": None, "xn": self.x,
            "k": d, "comb_w": self.comb_w, "cnt_local": self.cnt_local, "seg_rows": self.seg_rows, "cap": self.cap,
            "xq_off": self.off["xq"], "sf_off": self.off["xsf"], "rs_off": self.off["xrs"],
            "meta_off": self.off["meta"], "cnt_off": self.off["cnt"], "signal_site": DISP,
            "blk_expert": self.blk[0], "blk_row": self.blk[1], "blk_valid": self.blk[2], "num_blocks": self.blk[3],
            "row_list": self.row_list, "num_rows": self.num_rows, "err": self.err, "blk_rows": self.bn,
        }
        ops.ext().moe_dispatch_sp(args, slot, T)
        ops.ext().moe_owner_plan_sp(args, slot)
        blk = (self.blk[0], self.blk[1], self.blk[2], self.blk[3], self.max_blocks)
        w = self.w13
        ops.ext().gemm(w.packed, self.xq.packed, self.h, ops.EPI_SWIGLU, w.n, w.k, 0, self.bn, w.sf, self.xq.sf,
                       w.gscale, self.xq.row_scale, None, None, *blk, w.num_experts, 1 << 30, self.err, 0, 1, None,
                       None)
        ops.ext().quantize_rows_list(self.h, self.row_list, self.num_rows, self.hq.packed, self.hq.sf,
                                     self.hq.row_scale, 128, self.moe_rows)
        w = self.w2
        ops.ext().gemm(w.packed, self.hq.packed, self.h, ops.EPI_COMBINE_PUSH, w.n, w.k, 0, self.bn, w.sf, self.hq.sf,
                       w.gscale, self.hq.row_scale, None, None, *blk, w.num_experts, 1 << 30, self.err, 0, 1, None,
                       {"peer_slot": slot, "signal_site": COMB, "comb_off": self.off["comb"], "k_out": self.k,
                        "seg_rows": self.seg_rows, "cap": self.cap, "counts": self.cnt,
                        "meta": self.meta.data_ptr()})
        ops.ext().sp_land(self.xres, self.norm_w, 1e-6, False, T, LAND_COMB, OUT_LOCAL, None, 0, self.comb,
                          self.comb_w, self.k, self.xn, 0, 0, 0, 0, COMB, -1, slot, self.err)
        return self.xres

    # ------------------------------------------------------------------ NCCL baseline
    def nccl(self) -> torch.Tensor:
        T, d, k, N, E_l = self.T, self.d, self.k, self.N, self.E_l
        ops.linear_bf16(self.x, self.router_w, out=self.logits, epi=ops.EPI_STORE_F32)
        p = torch.softmax(self.logits[:, :self.E], -1)
        w, ids = torch.topk(p, k, -1)
        dest = (ids // E_l).flatten()
        order = torch.argsort(dest, stable=True)
        send = torch.bincount(dest, minlength=N)
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send)
        send_l, recv_l = send.tolist(), recv.tolist()  # split sizes: a host sync, as in any a2a dispatcher
        rows = self.x.index_select(0, order // k)
        eids = (ids.flatten() - dest * E_l)[order].to(torch.int32)
        R = sum(recv_l)
        rrows = torch.empty(R, d, dtype=torch.bfloat16, device=self.dev)
        reids = torch.empty(R, dtype=torch.int32, device=self.dev)
        dist.all_to_all_single(rrows, rows, recv_l, send_l)
        dist.all_to_all_single(reids, eids, recv_l, send_l)
        pl = self.plan_l
        pl.ids[:R, 0] = reids
        pl.weights[:R].fill_(1.0)
        pl.counts.copy_(torch.bincount(reids, minlength=E_l).to(torch.int32))
        ops.moe_plan(pl)
        ops.moe_dispatch_quantize(rrows, R, pl, self.xq_l)
        ops.grouped_nvfp4(self.xq_l, self.w13, self.h_l, ops.EPI_SWIGLU, pl, 128)
        ops.quantize_assigned(self.h_l, R, pl, self.hq_l)
        ops.grouped_nvfp4(self.hq_l, self.w2, self.y_l, ops.EPI_STORE_BF16, pl, 128)
        out_r = torch.empty(R, d, dtype=torch.bfloat16, device=self.dev)
        ops.moe_combine(self.y_l, pl, R, None, out_r)
        back = torch.empty(T * k, d, dtype=torch.bfloat16, device=self.dev)
        dist.all_to_all_single(back, out_r, send_l, recv_l)
        un = torch.empty_like(back)
        un[order] = back
        out = (un.view(T, k, d).float() * w.unsqueeze(-1)).sum(1).to(torch.bfloat16)
        self.stats = {"sent_rows": send_l, "recv_rows": R}
        return out


def _time(fn, par, flush, warmup, iters):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    tot = 0.0
    for _ in range(iters):
        flush.zero_()
        if dist.is_initialized():
            dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        tot += a.elapsed_time(b)
    return par.max_over_ranks(tot / iters)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--experts", type=int, default=128)
    ap.add_argument("--top-k", type=int, default=8)
    ap.add_argument("--inter", type=int, default=1536)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--profile", action="store_true", help="print a CUPTI per-kernel breakdown of both paths")
    ap.add_argument("--bn", type=int, default=128, choices=[128, 256], help="token tile of the fused GEMMs")
    a = ap.parse_args(argv)
    from .context import init_from_env
    par = init_from_env(timeout_s=120)
    N = par.world
    moe = EpMoE(par, a.tokens, a.hidden, a.experts, a.top_k, a.inter, bn=a.bn)
    ref = moe.nccl().float()
    got = moe.fused().float()
    ops.check_errors()
    cos = torch.nn.functional.cosine_similarity(got, ref, -1)
    cos_min = par.max_over_ranks(-float(cos.min()))
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=par.device)
    t_fused = _time(moe.fused, par, flush, a.warmup, a.iters)
    t_nccl = _time(moe.nccl, par, flush, a.warmup, a.iters)
    ops.check_errors()
    # ---- roofline of the fused path on this rank (then the max over ranks)
    moe.nccl()
    st = moe.stats
    d, k, inter = a.hidden, a.top_k, a.inter
    remote_out = sum(n for r, n in enumerate(st["sent_rows"]) if r != par.rank)
    row_q = d // 2 + d // 16 + 8                       # NVFP4 row + scales + row scale + slot meta
    nvl_bytes = remote_out * row_q + remote_out * d * 2  # dispatch pushes + combine pushes (out of this GPU)
    flops = 2.0 * st["recv_rows"] * (2 * inter * d + d * inter)
    peaks = {}
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))), "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            peaks = json.load(f)
    fp4_tflops = FP4_NOMINAL_TFLOPS * (peaks.get("bf16_tflops", 1590.0) / BF16_NOMINAL_TFLOPS)
    t_compute = flops / (fp4_tflops * 1e12) * 1e3
    t_link = nvl_bytes / (NVLINK_GBS * 1e9) * 1e3
    roof = par.max_over_ranks(max(t_compute, t_link)) if N > 1 else t_compute
    out = {
        "bench": "ep_moe", "n_gpus": N, "tokens_per_gpu": a.tokens, "hidden": d, "experts": a.experts,
        "experts_per_gpu": a.experts // N, "top_k": k, "inter": inter, "dtype": "nvfp4 weights, bf16 activations",
        "fused_bn": a.bn, "fused_ms": round(t_fused, 4), "nccl_ms": round(t_nccl, 4), "speedup_vs_nccl": round(t_nccl / t_fused, 3),
        "roofline_ms": round(roof, 4), "fused_frac_of_roofline": round(roof / t_fused, 3),
        "nvlink_bytes_out_per_gpu": int(nvl_bytes), "fp4_peak_tflops_scaled": round(fp4_tflops, 1),
        "tflops_fused": round(flops / (t_fused * 1e-3) / 1e12, 1), "min_row_cosine_fused_vs_nccl": round(-cos_min, 5),
        "timing": "CUDA events, L2 flushed between iterations, max over ranks",
    }
    if par.rank == 0:
        print(json.dumps(out), flush=True)
    if a.profile:
        from ..engine.profile import kernel_breakdown
        for name, fn in (("fused", moe.fused), ("nccl", moe.nccl)):
            br = kernel_breakdown(fn, reps=3, top=12)
            if par.rank == 0:
                print("KERNELS " + name + " " + json.dumps(br), flush=True)
    if N > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
