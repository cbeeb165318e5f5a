"""LLMEngine: the serving loop over one model replica (one process per GPU).

    engine = LLMEngine.from_fuel("glm-moe-355b", EngineConfig(...), random_init=True)
    outs = engine.generate([[1, 2, 3], ...], max_new_tokens=256)

Per step: the scheduler picks decode tokens + prefill chunks, the C++ KV
manager reserves slots, one packed int32 metadata buffer and the block table
go host->device (pinned, async), the model runs (a captured CUDA graph for a
pure-decode step of a bucketed batch size, eager otherwise) and the sampled
ids come back device->host.

Under tensor/expert parallelism every rank runs the same scheduler on the same
requests (rank 0's token decisions are broadcast so ranks never diverge: the
reference's rank-0-authoritative `sync_round_decision`,
engines/glm5-moe-nvfp4-2b/src/fabric/expert_parallel.h:100).
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field

import numpy as np
import torch

from .. import ops
from ..config import EngineConfig, ModelConfig, load_fuel
from ..models.moe_lm import MoELM
from ..parallel.context import ParallelCtx
from .scheduler import Request, Scheduler, ScheduledSeq, Status


@dataclass
class StepStats:
    steps: int = 0
    decode_steps: int = 0
    prefill_tokens: int = 0
    decode_tokens: int = 0
    graph_replays: int = 0
    h2d_bytes: int = 0
    d2h_bytes: int = 0
    step_ms: list = field(default_factory=list)


class LLMEngine:
    def __init__(self, model: MoELM, ecfg: EngineConfig, kv_pages: int | None = None,
                 memory_fraction: float | None = None):
        from .. import _rt  # C++ KV manager
        self.model = model
        self.cfg = model.cfg
        self.ecfg = ecfg
        self.par = model.par
        self.dev = model.dev
        ps = ecfg.page_size
        max_pages_per_seq = -(-ecfg.max_seq_len // ps)
        if kv_pages is None:
            free, _ = torch.cuda.mem_get_info(self.dev)
            frac = memory_fraction if memory_fraction is not None else ecfg.kv_memory_fraction
            kv_pages = int(free * frac) // model.kv_bytes_per_page()
        kv_pages = max(kv_pages, 2)
        # the last page is a scratch page for padded (dummy) decode rows; never handed out
        model.allocate_kv(kv_pages, max_pages_per_seq)
        self.dummy_page = kv_pages - 1
        # recurrent (DeltaNet) state cannot be rebuilt from cached KV pages: hybrid models run
        # without the prefix cache; every running request owns one recurrent-state slot
        self.hybrid = any(model.cfg.layer_kind(i) == "deltanet" for i in range(model.cfg.num_layers))
        self.kv = _rt.KvManager(kv_pages - 1, ps, max_pages_per_seq, bool(ecfg.prefix_cache) and not self.hybrid)
        self.free_slots = list(range(model.max_seqs - 1, -1, -1))
        self.dummy_slot = model.max_seqs  # recurrent-state slot written by padded decode rows
        self.slot_of: dict[int, int] = {}
        self.sched = Scheduler(self.kv, ecfg.max_batch, ecfg.prefill_chunk, ecfg.max_seq_len)
        self.stats = StepStats()
        m = model
        self.meta_len = 3 * m.max_tokens + 3 * m.max_seqs + 2 * m.max_work + 1 + 2 * m.max_seqs
        self.meta_dev = torch.zeros(self.meta_len, dtype=torch.int32, device=self.dev)
        self.meta_host = torch.zeros(self.meta_len, dtype=torch.int32).pin_memory()
        self.bt_host = torch.zeros(m.max_seqs, max_pages_per_seq, dtype=torch.int32).pin_memory()
        self.ids_host = torch.zeros(m.max_seqs, dtype=torch.int32).pin_memory()
        self._bind_meta()
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.kernels_per_decode_step: dict[int, int] = {}
        self.use_graphs = bool(ecfg.cuda_graphs)
        self.buckets = sorted(b for b in ecfg.batch_buckets if b <= min(m.max_decode, m.max_seqs))
        if self.par.world > 1:
            # sequence-parallel decode with fused collectives: buckets are multiples of the world size
            from ..models.sp_decode import SpDecode
            W = self.par.world
            self.buckets = sorted({-(-b // W) * W for b in self.buckets if -(-b // W) * W <= m.max_seqs})
            if ecfg.fused_collectives:
                model.sp = SpDecode(model, max(self.buckets) if self.buckets else ecfg.max_batch)
        # decode attention key splits for the largest bucket at the configured context
        if model.attn_index:
            sp = model.auto_decode_splits(max(self.buckets) if self.buckets else ecfg.max_batch, ecfg.max_seq_len)
            model.set_decode_splits(sp, max(ecfg.max_batch, 1))

    def _bind_meta(self):
        """Point the model's int32 step buffers at slices of one packed device buffer."""
        m = self.model
        T, S, Wm = m.max_tokens, m.max_seqs, m.max_work
        o = 0
        views = {}
        for name, n in (("ids", T), ("pos", T), ("slots", T), ("q_start", S), ("q_len", S), ("kv_len", S),
                        ("w_seq", Wm), ("w_tok0", Wm), ("num_work", 1), ("out_rows", S), ("state_slot", S)):
            views[name] = (o, n)
            o += n
        self.meta_off = views
        for name, (a, n) in views.items():
            setattr(m, name, self.meta_dev[a:a + n])

    # ------------------------------------------------------------------ public API
    @staticmethod
    def from_fuel(fuel: str, ecfg: EngineConfig, par: ParallelCtx | None = None, random_init: bool = True,
                  tensors: dict | None = None, seed: int = 0, kv_pages: int | None = None,
                  max_tokens: int | None = None, cfg_override: ModelConfig | None = None):
        cfg = cfg_override or load_fuel(fuel).model
        model = MoELM(cfg, par, max_tokens=max_tokens or ecfg.prefill_chunk, max_seqs=ecfg.max_batch,
                      max_decode=ecfg.max_batch, page_size=ecfg.page_size)
        if tensors is not None:
            model.load_fuel(tensors)
        else:
            model.init_random(seed)
        return LLMEngine(model, ecfg, kv_pages=kv_pages)

    def add_request(self, prompt, max_new_tokens: int, stop_ids=()) -> Request:
        r = Request(list(map(int, prompt)), max_new_tokens, tuple(stop_ids))
        self.sched.add(r)
        return r

    def generate(self, prompts, max_new_tokens: int = 128, stop_ids=()) -> list[list[int]]:
        reqs = [self.add_request(p, max_new_tokens, stop_ids) for p in prompts]
        while self.sched.has_work():
            self.step()
        return [r.output for r in reqs]

    # ------------------------------------------------------------------ one step
    def step(self) -> list[Request]:
        sched = self.sched.schedule()
        if not sched:
            if self.sched.has_work():
                raise RuntimeError("scheduler made no progress (KV pages exhausted?)")
            return []
        t0 = time.perf_counter()
        new_ids = self._run(sched)
        now = time.perf_counter()
        self.stats.step_ms.append((now - t0) * 1e3)
        self.stats.steps += 1
        done = self.sched.complete(sched, new_ids, now)
        for r in done:
            s = self.slot_of.pop(r.rid, None)
            if s is not None:
                self.free_slots.append(s)
        return done

    def _run(self, sched: list[ScheduledSeq]) -> np.ndarray:
        m = self.model
        decode = all(len(s.tokens) == 1 and s.req.status == Status.DECODE for s in sched)
        n = len(sched)
        B = n
        if decode and self.use_graphs:
            B = next((b for b in self.buckets if b >= n), n)
        T, S, w, n_out = self._stage(sched, B)
        if decode and self.use_graphs and B in self.buckets:
            g = self.graphs.get(B)
            if g is None:
                g = self._capture(B)
            g.replay()
            self.stats.graph_replays += 1
            out = m.out_ids[:n_out]
        else:
            out = m.forward(T, S, w, n_out, decode)
        if decode:
            self.stats.decode_steps += 1
            self.stats.decode_tokens += n
        else:
            self.stats.prefill_tokens += sum(len(s.tokens) for s in sched if s.req.status == Status.PREFILL)
        host = self.ids_host[:n_out]
        host.copy_(out, non_blocking=True)
        torch.cuda.current_stream(self.dev).synchronize()
        self.stats.d2h_bytes += n_out * 4
        res = host.numpy()[:n].copy()
        if self.par.world > 1:
            res = self._sync_decision(res)
        return res

    def _stage(self, sched: list[ScheduledSeq], B: int | None = None):
        """Reserve KV slots and stage one step's metadata on the device.
        Returns (T, S, work items, sampled rows)."""
        m = self.model
        n = len(sched)
        B = n if B is None else B
        meta = self.meta_host.numpy()
        o = self.meta_off
        ids = meta[o["ids"][0]:]
        pos = meta[o["pos"][0]:]
        slots = meta[o["slots"][0]:]
        qs = meta[o["q_start"][0]:]
        ql = meta[o["q_len"][0]:]
        kl = meta[o["kv_len"][0]:]
        ws = meta[o["w_seq"][0]:]
        wt = meta[o["w_tok0"][0]:]
        orow = meta[o["out_rows"][0]:]
        sslot = meta[o["state_slot"][0]:]
        bt = self.bt_host.numpy()
        G = max(1, m.Hq // m.Hkv)
        tpb = 128 // G
        t = 0
        w = 0
        n_out = 0
        seq_ids = []
        for i, s in enumerate(sched):
            r = s.req
            k = len(s.tokens)
            sl = self.kv.append(r.rid, s.tokens)
            ids[t:t + k] = s.tokens
            pos[t:t + k] = np.arange(s.start, s.start + k, dtype=np.int32)
            slots[t:t + k] = sl
            qs[i], ql[i], kl[i] = t, k, s.start + k
            if r.rid not in self.slot_of:
                self.slot_of[r.rid] = self.free_slots.pop()
            sslot[i] = self.slot_of[r.rid]
            for t0 in range(0, k, tpb):
                ws[w], wt[w] = i, t0
                w += 1
            if s.sample:
                orow[n_out] = t + k - 1
                n_out += 1
            seq_ids.append(r.rid)
            t += k
        self.kv.block_table(seq_ids, bt[:n])
        # pad a decode batch to its bucket with dummy rows on the scratch page
        for i in range(n, B):
            ids[t] = 0
            pos[t] = 0
            slots[t] = self.dummy_page * self.ecfg.page_size
            qs[i], ql[i], kl[i] = t, 1, 1
            sslot[i] = self.dummy_slot
            ws[w], wt[w] = i, 0
            w += 1
            orow[n_out] = t
            n_out += 1
            bt[i, 0] = self.dummy_page
            t += 1
        meta[o["num_work"][0]] = w
        T, S = t, B
        # host -> device: one packed metadata copy + the block-table rows in use
        self.meta_dev.copy_(self.meta_host, non_blocking=True)
        m.block_table[:S].copy_(self.bt_host[:S], non_blocking=True)
        self.stats.h2d_bytes += self.meta_len * 4 + S * bt.shape[1] * 4
        return T, S, w, n_out

    def prompt_logits(self, prompt) -> torch.Tensor:
        """fp32 logits (this rank's vocab shard) after prefilling `prompt` in one
        eager step; the sequence is freed afterwards.  Numerics/debug API."""
        r = Request(list(map(int, prompt)), 1)
        self.kv.open(r.rid, [])
        r.status = Status.PREFILL
        m = self.model
        if not hasattr(self, "_dbg_logits"):
            self._dbg_logits = torch.zeros(m.max_seqs, m.V_l, dtype=torch.float32, device=self.dev)
        s = ScheduledSeq(r, r.prompt, 0, True)
        self._stage([s])
        meta = self.meta_host.numpy()
        w = int(meta[self.meta_off["num_work"][0]])
        lg = m.forward(len(r.prompt), 1, w, 1, False, logits_out=self._dbg_logits)
        out = lg[0, : min(m.V_l, self.cfg.vocab_size - m.v_lo)].float().cpu()
        self.kv.free(r.rid)
        s = self.slot_of.pop(r.rid, None)
        if s is not None:
            self.free_slots.append(s)
        return out

    def _sync_decision(self, ids: np.ndarray) -> np.ndarray:
        t = torch.from_numpy(ids).to(self.dev)
        self.par.broadcast(t, 0)
        return t.cpu().numpy()

    def _capture(self, B: int) -> torch.cuda.CUDAGraph:
        """Capture one decode step of batch B (metadata already staged)."""
        m = self.model
        torch.cuda.synchronize(self.dev)
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            m.forward(B, B, B, B, True)  # warm-up launch outside the graph
        torch.cuda.current_stream(self.dev).wait_stream(s)
        torch.cuda.synchronize(self.dev)
        g = torch.cuda.CUDAGraph()
        n0 = ops.launch_count()
        with torch.cuda.graph(g, stream=s):
            m.forward(B, B, B, B, True)
        self.kernels_per_decode_step[B] = ops.launch_count() - n0
        torch.cuda.synchronize(self.dev)
        self.graphs[B] = g
        return g

    def release_graphs(self):
        self.graphs.clear()
        torch.cuda.synchronize(self.dev)

    # ------------------------------------------------------------------ metrics
    @staticmethod
    def latency_summary(reqs: list[Request]) -> dict:
        ttft = sorted((r.t_first - r.arrival) * 1e3 for r in reqs if r.t_first)
        itl = []
        for r in reqs:
            itl += [(b - a) * 1e3 for a, b in zip(r.t_tokens, r.t_tokens[1:])]
        itl.sort()
        p = lambda a, q: a[min(len(a) - 1, int(q * len(a)))] if a else None
        return {"ttft_ms_p50": p(ttft, 0.5), "ttft_ms_p95": p(ttft, 0.95), "itl_ms_p50": p(itl, 0.5),
                "itl_ms_p95": p(itl, 0.95)}
