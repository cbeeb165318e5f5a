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

import os
import time
from dataclasses import dataclass, field

import numpy as np
import torch

from .. import ops
from ..config import EngineConfig, ModelConfig, load_fuel
from ..models.moe_lm import MoELM
from ..parallel.context import ParallelCtx
from .scheduler import Request, Scheduler, ScheduledSeq, SeqResult, Status


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


class EngineFaulted(RuntimeError):
    """A step raised earlier; the engine refuses further steps."""


class SchedulerStall(RuntimeError):
    """No request could be scheduled (KV pages exhausted): nothing ran on the device, so the
    engine stays usable once requests are aborted or pages freed."""


@dataclass
class Detached:
    """A request parked by LLMEngine.detach: KV pages on the device, recurrent state
    (DeltaNet state, conv taps) in host memory."""
    req: Request
    state: tuple | None = None


def sharded_token_nll(lg: torch.Tensor, tgt: torch.Tensor, v_lo: int, par) -> torch.Tensor:
    """-log softmax(logits)[target] per row when each rank holds the logit columns
    [v_lo, v_lo + lg.shape[1]) of the vocabulary: all-reduce(max) of the row maxima,
    then one all-reduce(sum) of the shifted exp-sums and of the target logit (from the
    rank that owns it)."""
    n = lg.shape[1]
    mx = lg.max(-1).values if n else torch.full((lg.shape[0],), -float("inf"), device=lg.device)
    par.all_reduce_max(mx)
    se = torch.exp(lg - mx[:, None]).sum(-1) if n else torch.zeros_like(mx)
    loc = tgt - v_lo
    mine = (loc >= 0) & (loc < n)
    t_logit = (torch.where(mine, lg.gather(1, loc.clamp(0, n - 1)[:, None])[:, 0], torch.zeros_like(mx))
               if n else torch.zeros_like(mx))
    both = torch.stack([se, t_logit])
    par.all_reduce(both)
    return mx + torch.log(both[0]) - both[1]


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
        self.K = model.spec_k
        # speculative steps write up to 2K positions past the committed length
        max_pages_per_seq = -(-(ecfg.max_seq_len + 2 * self.K) // ps)
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
        self.sched = Scheduler(self.kv, ecfg.max_batch, ecfg.prefill_chunk, ecfg.max_seq_len, self.K)
        self.drafts = None
        if self.K and ecfg.draft_source:
            self.set_draft_source(ecfg.draft_source, ecfg.draft_file or None)
        if self.K and not model.has_mtp and self.drafts is None:
            raise ValueError("speculative decoding on a model without an MTP head needs a host draft source "
                             "(draft_source prompt_lookup, history or file)")
        # speculation depth of each step (MTP draft passes; the next step verifies that many)
        self.depth_policy = None
        if ecfg.spec_depth not in ("fixed", "adaptive"):
            raise ValueError(f"spec_depth={ecfg.spec_depth!r}: fixed | adaptive")
        if self.K and ecfg.spec_depth == "adaptive":
            if not model.has_mtp:
                raise ValueError("adaptive speculation depth adapts the MTP chain: the model has no MTP head")
            from .depth import DepthPolicy
            self.depth_policy = DepthPolicy(self.K)
        self.k_step = self.K   # drafts this step produces
        self.k_next = self.K   # ... the next step produces (rank 0's decision, broadcast with the results)
        self.v_width = self.K  # drafts the next verify feeds (what the previous step produced)
        self.stats = StepStats()
        from ..utils.metrics import Metrics
        self.metrics = Metrics(labels={"rank": self.par.rank})
        self.health = None  # parallel.health.Health (multi-rank serving; see enable_health)
        from ..utils.tracing import NULL_TRACER
        self.tracer = NULL_TRACER  # utils.tracing.Tracer when attached (host spans)
        # execution state: idle between steps, active inside one, faulted after a step raised
        # (terminal: device buffers and peer ranks may be mid-step; build a new engine)
        self.phase = "idle"
        self.fault: str | None = None
        from ..utils.checksums import ChecksumTap
        self.checksums = ChecksumTap.from_env(self)  # ROCKET_CHECKSUM=kv,hidden,spec debug taps
        m = model
        self.meta_len = 3 * m.max_tokens + 3 * m.max_seqs + 2 * m.max_work + 1 + m.max_out + m.max_seqs
        if self.K:
            self.meta_len += 2 * m.max_seqs + 2 * m.max_tokens  # verify, sample, out_idx, next_tok
        self.meta_dev = torch.zeros(self.meta_len, dtype=torch.int32, device=self.dev)
        self.meta_host = torch.zeros(self.meta_len, dtype=torch.int32).pin_memory()
        self._py_stage = os.environ.get("ROCKET_PY_STAGE", "0") == "1"
        self.bt_host = torch.zeros(m.max_seqs, max_pages_per_seq, dtype=torch.int32).pin_memory()
        self.out_host = torch.zeros(m.step_out.numel(), dtype=torch.int32).pin_memory()
        self._bind_meta()
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.kernels_per_decode_step: dict[int, int] = {}
        # streamed experts and the sentinel check read back to the host: eager steps only
        self.use_graphs = bool(ecfg.cuda_graphs) and model.streamer is None and not model.sentinel
        self.buckets = sorted(b for b in ecfg.batch_buckets if b <= min(m.max_decode, m.max_seqs))
        if ecfg.collectives not in ("fused", "sp", "nccl"):
            raise ValueError(f"collectives={ecfg.collectives!r}: fused | sp | nccl")
        if self.par.world > 1:
            # the fused paths keep one residual stream, GQA attention and resident experts
            simple = (not model.hc and model.cfg.sparse_attention is None and model.cfg.mla is None
                      and model.streamer is None and not self.hybrid)
            if ecfg.collectives == "sp" and simple and not model.cfg.attention_bias:
                # sequence-parallel decode with fused collectives: buckets are multiples of the world size
                from ..models.sp_decode import SpDecode
                W = self.par.world
                self.buckets = sorted({-(-b // W) * W for b in self.buckets if -(-b // W) * W <= m.max_seqs})
                model.sp = SpDecode(model, max(self.buckets) if self.buckets else ecfg.max_batch)
            elif ecfg.collectives == "fused" and simple and self._fused_syncs(model) >= 2:
                # replicated tokens, all-reduce / combine pushed from the GEMM epilogues; with
                # attention replicated (tp = 1) every step runs it (exact single-GPU parity),
                # otherwise decode steps do and prefill chunks use NCCL
                from ..models.ar_decode import ArFused
                rows = m.max_tokens if self.par.tp == 1 else max(self.buckets or [ecfg.max_batch])
                model.ar = ArFused(model, rows)
        # decode attention key splits for the largest bucket at the configured context
        if model.attn_index:
            model.configure_attention(max(self.buckets) if self.buckets else ecfg.max_batch, ecfg.max_seq_len)

    @staticmethod
    def _fused_syncs(model) -> int:
        """Cross-rank syncs of one replicated-token fused step: the attention all-reduce under
        TP > 1, and the MoE combine or the dense all-reduce under TP > 1.  Its rotating
        buffers need at least two per step (see models/ar_decode.py)."""
        c, par = model.cfg, model.par
        return sum(int(par.tp > 1) + int(c.is_moe_layer(i) or par.tp > 1) for i in range(c.num_layers))

    def _bind_meta(self):
        """Point the model's int32 step buffers at slices of one packed device buffer."""
        m = self.model
        T, S, Wm = m.max_tokens, m.max_seqs, m.max_work
        o = 0
        views = {}
        fields = [("ids", T), ("pos", T), ("slots", T), ("q_start", S), ("q_len", S), ("kv_len", S),
                  ("w_seq", Wm), ("w_tok0", Wm), ("num_work", 1), ("out_rows", m.max_out), ("state_slot", S)]
        if self.K:
            fields += [("verify", S), ("sample", S), ("out_idx", T), ("next_tok", T)]
        for name, n in fields:
            views[name] = (o, n)
            o += n
        self.meta_off = views
        for name, (a, n) in views.items():
            setattr(m, name, self.meta_dev[a:a + n])

    # ------------------------------------------------------------------ public API
    @staticmethod
    def from_fuel(fuel: str, ecfg: EngineConfig, par: ParallelCtx | None = None, random_init: bool = True,
                  tensors: dict | None = None, seed: int = 0, kv_pages: int | None = None,
                  max_tokens: int | None = None, cfg_override: ModelConfig | None = None,
                  fuel_dir: str | None = None, expert_order: list[int] | None = None,
                  verify_checksums: bool = False, expert_slab: str | None = None):
        """Engine for fuel `fuel` (a name under rocket_b200/fuels or a fuel.yaml path).
        Weights: `tensors` (fuel-format CPU tensors), else the safetensors checkpoint in
        `fuel_dir`, else random init on the device."""
        cfg = cfg_override or load_fuel(fuel).model
        if fuel_dir is not None:
            from ..config.hf import check_checkpoint_dir
            check_checkpoint_dir(cfg, fuel_dir)  # a config.json that disagrees with the fuel is refused
        if tensors is None and fuel_dir is not None:
            from ..fuel.safetensors_io import load_dir
            if verify_checksums:
                from ..fuel.materialize import verify
                bad = verify(fuel_dir)
                if bad:
                    raise ValueError(f"{fuel_dir}: shard digest mismatch: {bad}")
            tensors = load_dir(fuel_dir)
        # a speculative verify feeds K+1 rows per sequence
        max_tokens = max(max_tokens or ecfg.prefill_chunk, (ecfg.spec_tokens + 1) * ecfg.max_batch)
        if par is not None and par.world > 1:
            par = par.with_layout(ecfg.tp, ecfg.ep)
        model = MoELM(cfg, par, max_tokens=max_tokens, max_seqs=ecfg.max_batch,
                      max_decode=ecfg.max_batch, page_size=ecfg.page_size, spec_tokens=ecfg.spec_tokens,
                      expert_order=expert_order, kv_dtype=ecfg.kv_dtype)
        if ecfg.expert_cache_slots:
            model.enable_expert_streaming(ecfg.expert_cache_slots)
        if tensors is not None:
            if expert_slab and os.path.isdir(expert_slab):
                from ..fuel.slabs import slab_name
                expert_slab = os.path.join(expert_slab, slab_name(model.par.ep_rank, model.par.ep))
            model.load_fuel(tensors, expert_slab=expert_slab)
        else:
            model.init_random(seed)
        return LLMEngine(model, ecfg, kv_pages=kv_pages)

    def add_request(self, prompt, max_new_tokens: int, stop_ids=()) -> Request:
        r = Request(list(map(int, prompt)), max_new_tokens, tuple(stop_ids))
        self.sched.add(r)
        self.metrics.inc("requests_total")
        self.metrics.inc("prompt_tokens_total", len(r.prompt))
        return r

    def generate(self, prompts, max_new_tokens: int = 128, stop_ids=()) -> list[list[int]]:
        reqs = [self.add_request(p, max_new_tokens, stop_ids) for p in prompts]
        while self.sched.has_work():
            self.step()
        return [r.output for r in reqs]

    def abort(self, req: Request):
        """Drop a request (running or waiting): its KV pages and state slot are freed."""
        if req in self.sched.waiting:
            self.sched.waiting.remove(req)
            return
        if req in self.sched.running:
            self.sched.running.remove(req)
            self.kv.free(req.rid)
        req.status = Status.FINISHED
        if self.drafts is not None:
            self.drafts.release(req)
        s = self.slot_of.pop(req.rid, None)
        if s is not None:
            self.free_slots.append(s)

    def fork(self, parent: Request, max_new_tokens: int, stop_ids=None) -> Request:
        """A new request that continues from `parent`'s current state: the same tokens so
        far (prompt and output are copied), its KV pages shared (the partially filled
        boundary page is copied so both can extend it), its recurrent DeltaNet state and
        its drafts copied.  The child then decodes up to `max_new_tokens` more tokens on
        its own.  Call between steps on a decoding request; under tensor parallelism
        every rank calls it in the same order.

        Counterpart of the reference engine's kv_fork (engines/glm5-moe-nvfp4-2b/src/
        model.cu:930) over the paged KV manager's fork (kv/page_pool.cc)."""
        if parent.status != Status.DECODE or parent not in self.sched.running:
            raise ValueError("fork needs a running, decoding request")
        if len(self.sched.running) >= self.sched.max_batch or not self.free_slots:
            raise RuntimeError("fork: the batch is full")
        m = self.model
        child = Request(list(parent.prompt), len(parent.output) + int(max_new_tokens),
                        tuple(parent.stop_ids if stop_ids is None else stop_ids))
        child.output = list(parent.output)
        if len(child.prompt) + child.max_new_tokens > self.sched.max_seq_len:
            raise ValueError(f"fork: {len(child.prompt) + child.max_new_tokens} tokens > max_seq_len "
                             f"{self.sched.max_seq_len}")
        need = self.kv.pages_needed(parent.rid, int(max_new_tokens) + 2 * self.K) + 1
        if need > self.kv.num_free_pages():
            raise RuntimeError("fork: not enough free KV pages")
        copies = self.kv.fork(parent.rid, child.rid)
        caches = [c for c in m.page_caches() if c.numel()]
        for op in copies:
            for c in caches:
                c[:, op.dst].copy_(c[:, op.src])
        slot = self.free_slots.pop()
        self.slot_of[child.rid] = slot
        if self.hybrid:
            b = m.dn_buf
            ps = self.slot_of[parent.rid]
            b.state[:, slot].copy_(b.state[:, ps])
            b.conv_state[:, slot].copy_(b.conv_state[:, ps])
        child.computed = parent.computed
        child.drafts = list(parent.drafts)
        child.status = Status.DECODE
        child.t_first = child.arrival
        self.sched.running.append(child)
        self.metrics.inc("requests_total")
        return child

    def detach(self, req: Request) -> "Detached":
        """Park a decoding request between steps: it leaves the batch and its recurrent-state
        slot (DeltaNet state and conv taps move to pinned host memory), while its KV pages
        stay allocated on the device, so `attach` resumes it without recomputing anything.
        For idle sessions (an agent waiting on a tool) that must not hold a batch slot.

        Counterpart of the reference engine's detach / resume (engines/glm5-moe-nvfp4-2b/
        src/model.h:155-190, HostKdaStateStore in kv/kv_arena.h:94)."""
        if req.status != Status.DECODE or req not in self.sched.running:
            raise ValueError("detach needs a running, decoding request")
        state = None
        slot = self.slot_of.pop(req.rid, None)
        if slot is not None:
            if self.hybrid:
                b = self.model.dn_buf
                pin = torch.cuda.is_available()
                state = tuple(torch.empty(t[:, slot].shape, dtype=t.dtype, pin_memory=pin).copy_(t[:, slot])
                              for t in (b.state, b.conv_state))
            self.free_slots.append(slot)
        self.sched.running.remove(req)
        return Detached(req, state)

    def attach(self, d: "Detached") -> Request:
        """Resume a request parked by `detach` (its KV pages never left the device)."""
        req = d.req
        if len(self.sched.running) >= self.sched.max_batch or not self.free_slots:
            raise RuntimeError("attach: the batch is full")
        slot = self.free_slots.pop()
        self.slot_of[req.rid] = slot
        if self.hybrid and d.state is not None:
            b = self.model.dn_buf
            b.state[:, slot].copy_(d.state[0].to(b.state.device, non_blocking=True))
            b.conv_state[:, slot].copy_(d.state[1].to(b.conv_state.device, non_blocking=True))
        self.sched.running.append(req)
        return req

    def drop(self, d: "Detached"):
        """Discard a parked request: its KV pages are freed."""
        self.kv.free(d.req.rid)
        d.req.status = Status.FINISHED
        if self.drafts is not None:
            self.drafts.release(d.req)

    def set_draft_source(self, spec, draft_file: str | None = None, draft_engine=None):
        """Host draft sources for the verify steps (engine.drafts): a '+'-joined priority
        list such as 'prompt_lookup+mtp' or 'draft_model' (with `draft_engine`, an
        LLMEngine of a smaller model with the same vocabulary), or a DraftSource object.
        'mtp' restores the device MTP chain alone."""
        from .drafts import DraftSource, make_draft_source
        if not self.K:
            raise ValueError("draft sources need speculative decoding (spec_tokens > 0)")
        src = spec if isinstance(spec, DraftSource) else make_draft_source(spec, draft_file, draft_engine)
        for s in getattr(src, "sources", [src]):
            v = getattr(s, "vocab_size", None)
            if v is not None and v != self.cfg.vocab_size:
                raise ValueError(f"draft model vocabulary {v} != target vocabulary {self.cfg.vocab_size}")
        if src is None and not self.model.has_mtp:
            raise ValueError("the model has no MTP head: pick a host draft source (prompt_lookup, history, file)")
        self.drafts = src
        K = self.K
        self.sched.draft_hook = (lambda r: src.propose(r, K)) if src is not None else None

    def attach_prefix_tier(self, tier):
        """Back the GPU prefix cache with a persistent tier (kv.prefix_store.PrefixTier)."""
        if self.hybrid or not self.kv.prefix_cache():
            raise ValueError("the prefix tier needs the prefix cache (attention-only models)")
        self.prefix_tier = tier
        self.sched.before_open = tier.restore
        self.sched.after_commit = tier.save

    def enable_health(self, **kw):
        """Start host-side failure detection (heartbeats + failure markers in a TCPStore
        next to the process group's).  Every step checks it before launching kernels."""
        if self.par.world > 1 and self.health is None:
            from ..parallel.health import from_env
            self.health = from_env(self.par.rank, self.par.world, **kw)
        return self.health

    # ------------------------------------------------------------------ one step
    def step(self) -> list[Request]:
        if self.phase == "faulted":
            raise EngineFaulted(f"engine faulted in an earlier step ({self.fault}); build a new engine")
        if self.health is not None:
            self.health.check()  # a failed peer surfaces here, before any launch of this step
        self.phase = "active"
        try:
            with self.tracer.span("step", phase="step"):
                out = self._step()
            self.phase = "idle"
            return out
        except SchedulerStall:
            self.phase = "idle"  # raised before any launch of this step
            raise
        except Exception as e:
            self.phase = "faulted"
            self.fault = f"{type(e).__name__}: {e}"
            if self.health is not None:
                self.health.fail(self.fault)
            raise

    def _step(self) -> list[Request]:
        if self.drafts is not None and hasattr(self.drafts, "prepare"):
            with self.tracer.span("drafts", phase="host"):
                self.drafts.prepare(self.sched.running, self.K)
        if self.depth_policy is not None:
            self.k_step = self.k_next
            self.sched.verify_width = self.v_width
        with self.tracer.span("schedule", phase="host"):
            sched = self.sched.schedule()
        if not sched:
            if self.sched.has_work():
                raise SchedulerStall("scheduler made no progress (KV pages exhausted?)")
            return []
        t0 = time.perf_counter()
        replays0 = self.stats.graph_replays
        decode = all(s.req.status == Status.DECODE for s in sched)
        with self.tracer.span("run", phase="decode" if decode else "mixed", bucket=len(sched)):
            results = self._run(sched)
        if self.checksums is not None:
            self.checksums.after_step(sched, self._last_T)
        now = time.perf_counter()
        self.stats.step_ms.append((now - t0) * 1e3)
        self.stats.steps += 1
        before = [(len(s.req.output), s.req.t_first, s.req.t_tokens[-1] if s.req.t_tokens else None) for s in sched]
        if self.depth_policy is not None:
            if decode:
                acc = [max(0, len(res.tokens) - 1) for s, res in zip(sched, results) if s.verify]
                self.depth_policy.observe(self.v_width, self.k_step, acc, (now - t0) * 1e3)
            self.v_width = self.k_step
        done = self.sched.complete(sched, results, now)
        self._observe(sched, before, results, (now - t0) * 1e3, self.stats.graph_replays - replays0)
        for r in done:
            s = self.slot_of.pop(r.rid, None)
            if s is not None:
                self.free_slots.append(s)
            if self.drafts is not None:
                self.drafts.release(r)
        return done

    def _observe(self, sched, before, results, step_ms, replays):
        mt = self.metrics
        mt.inc("steps_total")
        mt.inc("graph_replays_total", replays)
        mt.observe("step_ms", step_ms)
        for s, (n0, tf0, tl0), res in zip(sched, before, results):
            r = s.req
            new = len(r.output) - n0
            mt.inc("generated_tokens_total", new)
            if s.verify:
                mt.inc("spec_drafted_total", len(s.tokens) - 1)
                mt.inc("spec_accepted_total", max(0, len(res.tokens) - 1))
            if tf0 is None and r.t_first is not None:
                mt.observe("ttft_ms", (r.t_first - r.arrival) * 1e3)
            elif new and tl0 is not None:
                mt.observe("itl_ms", (r.t_tokens[-1] - tl0) * 1e3 / new)
        mt.set("running_requests", len(self.sched.running))
        mt.set("waiting_requests", len(self.sched.waiting))
        mt.set("free_kv_pages", self.kv.num_free_pages())
        mt.c["prefix_lookups_total"] = int(self.kv.lookups())
        mt.c["prefix_hits_total"] = int(self.kv.hits())
        st = self.model.streamer
        if st is not None:  # streamed experts: slot-cache counters
            ex = st.stats()
            mt.c["expert_slot_hits_total"] = int(ex["hits"])
            mt.c["expert_slot_misses_total"] = int(ex["misses"])
            mt.c["expert_bytes_streamed_total"] = int(ex["bytes_loaded"])

    def _run(self, sched: list[ScheduledSeq]) -> list[SeqResult]:
        m = self.model
        K = self.K
        if K:
            # verify sequences first: their rows [0, spec_rows) are the ones DeltaNet retains
            sched.sort(key=lambda s: not s.verify)
        decode = all(s.req.status == Status.DECODE for s in sched)
        n = len(sched)
        B = n
        if decode and self.use_graphs:
            B = next((b for b in self.buckets if b >= n), n)
        T, S, w, n_out = self._stage(sched, B)
        self._last_T = T
        graphed = decode and self.use_graphs and B in self.buckets
        key = ("spec", B, self._width(), self._passes()) if K else B
        if graphed:
            g = self.graphs.get(key)
            if g is None:
                g = self._capture(B, T, w, n_out)
            g.replay()
            self.stats.graph_replays += 1
        elif K:
            n_verify = sum(1 for s in sched if s.verify) + (B - n if decode else 0)
            m.spec_forward(T, S, w, n_out, self._spec_rows(sched, B), n_verify, self.dummy_page,
                           draft_passes=self._passes())
        else:
            m.forward(T, S, w, n_out, decode)
        if decode:
            self.stats.decode_steps += 1
        else:
            self.stats.prefill_tokens += sum(len(s.tokens) for s in sched if s.req.status == Status.PREFILL)
        # device -> host: one packed copy of the step's outputs
        n_copy = n_out if not K else m.step_out.numel()
        host = self.out_host[:n_copy]
        host.copy_(m.step_out[:n_copy], non_blocking=True)
        torch.cuda.current_stream(self.dev).synchronize()
        self.stats.d2h_bytes += n_copy * 4
        res = host.numpy().copy()
        if self.depth_policy is not None:
            # the next step's depth: rank 0 decides (on observations up to the previous step)
            # and every rank takes it from the same broadcast as the tokens
            nxt = self.depth_policy.decide() if self.par.rank == 0 else 0
            res = np.append(res, np.int32(nxt))
        if self.par.world > 1:
            res = self._sync_decision(res)
        if self.depth_policy is not None:
            self.k_next = int(res[-1])
            res = res[:-1]
        return self._results(sched, res, S)

    def _width(self) -> int:
        """Drafts each verify sequence feeds this step."""
        w = getattr(getattr(self, "sched", None), "verify_width", None)
        return self.K if w is None else w

    def _passes(self) -> int:
        """MTP draft passes (next drafts) of this step."""
        return getattr(self, "k_step", self.K)

    def _spec_rows(self, sched, B) -> int:
        rows = sum(len(s.tokens) for s in sched if s.verify)
        return rows + (B - len(sched)) * (self._width() + 1)

    def _results(self, sched, res, S) -> list[SeqResult]:
        """Per-sequence emitted tokens / committed KV length / next drafts."""
        m = self.model
        K = self.K
        out = []
        k = 0
        for i, s in enumerate(sched):
            if not s.sample:
                out.append(SeqResult([], s.start + len(s.tokens) if s.reserve else None))
                continue
            if not K:
                out.append(SeqResult([int(res[k])]))
                k += 1
                continue
            Smax = m.max_seqs  # drafts are [K][max_seqs] in the packed output; this step made k_step
            drafts = [int(res[m.max_out + Smax + j * Smax + i]) for j in range(self._passes())] if m.has_mtp else []
            if s.verify:
                a = int(res[m.max_out + i])
                toks = [int(t) for t in res[k:k + a + 1]]
                k += len(s.tokens)
                self.stats.decode_tokens += len(toks)
                out.append(SeqResult(toks, s.start + a + 1, drafts))
            else:
                out.append(SeqResult([int(res[k])], s.start + len(s.tokens), drafts))
                k += 1
        if not K:
            self.stats.decode_tokens += sum(len(r.tokens) for r, s in zip(out, sched) if s.req.status == Status.DECODE)
        return out

    def _stage(self, sched: list[ScheduledSeq], B: int | None = None):
        """Reserve KV slots and stage one step's metadata on the device.
        Returns (T, S, work items, sampled rows).

        The metadata is written by the C++ stager (runtime/stager.cc) in one call;
        ROCKET_PY_STAGE=1 selects the Python restatement below, which defines the
        field semantics the native code is tested against."""
        m = self.model
        K = self.K
        n = len(sched)
        B = n if B is None else B
        if not self._py_stage:
            return self._stage_native(sched, B)
        meta = self.meta_host.numpy()
        o = self.meta_off
        v = lambda name: meta[o[name][0]:o[name][0] + o[name][1]]
        ids, pos, slots, qs, ql, kl = v("ids"), v("pos"), v("slots"), v("q_start"), v("q_len"), v("kv_len")
        ws, wt, orow, sslot = v("w_seq"), v("w_tok0"), v("out_rows"), v("state_slot")
        if K:
            ver, smp, oidx, ntok = v("verify"), v("sample"), v("out_idx"), v("next_tok")
        bt = self.bt_host.numpy()
        G = max(1, m.Hq // m.Hkv)
        tpb = 128 // G
        t = 0
        w = 0
        n_out = 0
        seq_ids = []
        ps = self.ecfg.page_size
        for i, s in enumerate(sched):
            r = s.req
            k = len(s.tokens)
            sl = self.kv.append(r.rid, s.tokens + [0] * s.reserve)
            ids[t:t + k] = s.tokens
            pos[t:t + k] = np.arange(s.start, s.start + k, dtype=np.int32)
            slots[t:t + k] = sl[:k]
            qs[i], ql[i], kl[i] = t, k, s.start + k
            if r.rid not in self.slot_of:
                self.slot_of[r.rid] = self.free_slots.pop()
            sslot[i] = self.slot_of[r.rid]
            for t0 in range(0, k, tpb):
                ws[w], wt[w] = i, t0
                w += 1
            if K:
                ver[i], smp[i] = int(s.verify), int(s.sample)
                oidx[t:t + k] = -1
                if s.verify:
                    orow[n_out:n_out + k] = np.arange(t, t + k)
                    oidx[t:t + k] = np.arange(n_out, n_out + k)
                    ntok[t:t + k] = -1
                    n_out += k
                else:
                    # prefill rows: the next prompt token; the last prompt row takes the sampled token
                    nxt = r.prompt[s.start + 1:s.start + k + 1]
                    ntok[t:t + len(nxt)] = nxt
                    ntok[t + len(nxt):t + k] = -1
                    if s.sample:
                        orow[n_out] = t + k - 1
                        oidx[t + k - 1] = n_out
                        n_out += 1
            elif s.sample:
                orow[n_out] = t + k - 1
                n_out += 1
            seq_ids.append(r.rid)
            t += k
        self.kv.block_table(seq_ids, bt[:n])
        # pad a decode batch to its bucket with dummy sequences on the scratch page
        rows = self._width() + 1 if K else 1
        for i in range(n, B):
            ids[t:t + rows] = 0
            pos[t:t + rows] = np.arange(rows)
            slots[t:t + rows] = self.dummy_page * ps + np.arange(rows)
            qs[i], ql[i], kl[i] = t, rows, rows
            sslot[i] = self.dummy_slot
            for t0 in range(0, rows, tpb):
                ws[w], wt[w] = i, t0
                w += 1
            orow[n_out:n_out + rows] = np.arange(t, t + rows)
            if K:
                ver[i], smp[i] = 1, 1
                oidx[t:t + rows] = np.arange(n_out, n_out + rows)
                ntok[t:t + rows] = -1
            n_out += rows
            bt[i, 0] = self.dummy_page
            t += rows
        meta[o["num_work"][0]] = w
        T, S = t, B
        # host -> device: one packed metadata copy + the block-table rows in use
        self.meta_dev.copy_(self.meta_host, non_blocking=True)
        m.block_table[:S].copy_(self.bt_host[:S], non_blocking=True)
        self.stats.h2d_bytes += self.meta_len * 4 + S * bt.shape[1] * 4
        return T, S, w, n_out

    def _stage_native(self, sched: list[ScheduledSeq], B: int):
        from .. import _rt
        m = self.model
        K = self.K
        items = []
        for s in sched:
            r = s.req
            if r.rid not in self.slot_of:
                self.slot_of[r.rid] = self.free_slots.pop()
            nxt = r.prompt[s.start + 1:s.start + len(s.tokens) + 1] if (K and not s.verify) else []
            items.append((r.rid, s.tokens, s.start, int(s.sample), int(s.verify), s.reserve,
                          self.slot_of[r.rid], nxt))
        bt = self.bt_host.numpy()
        T, S, w, n_out = _rt.stage_step(self.kv, items, B, K, 128 // max(1, m.Hq // m.Hkv), self.ecfg.page_size,
                                        self.dummy_page, self.dummy_slot, self.meta_off, self.meta_host.numpy(), bt,
                                        self._width() + 1 if K else 1)
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

    def mtp_prompt_logits(self, prompt) -> tuple[int, torch.Tensor]:
        """Prefill `prompt` in one eager speculative step; returns the target's next token
        y and the fp32 logits (this rank's vocab shard) of the MTP head at the last prompt
        row (hidden state of that row paired with y).  Numerics/debug API."""
        if not self.K or not self.model.has_mtp:
            raise ValueError("engine built without an MTP head")
        r = Request(list(map(int, prompt)), 1)
        self.kv.open(r.rid, [])
        r.status = Status.PREFILL
        m = self.model
        if not hasattr(self, "_dbg_logits"):
            self._dbg_logits = torch.zeros(m.max_seqs, m.V_l, dtype=torch.float32, device=self.dev)
        s = ScheduledSeq(r, r.prompt, 0, True, reserve=self.K - 1)
        T, S, w, n_out = self._stage([s])
        lg = m.spec_forward(T, S, w, n_out, 0, 0, self.dummy_page, mtp_logits_out=self._dbg_logits)
        y = int(m.out_ids[0].item())
        out = lg[0, : min(m.V_l, self.cfg.vocab_size - m.v_lo)].float().cpu()
        self.kv.free(r.rid)
        sl = self.slot_of.pop(r.rid, None)
        if sl is not None:
            self.free_slots.append(sl)
        return y, out

    def teacher_score(self, seq: list[int]) -> list[int]:
        """Teacher-forced greedy predictions: the argmax next token after every prefix of
        `seq` (len(seq) ids; the last one predicts past the end).  Runs `seq` as eager
        prefill chunks whose every row is sampled; the sequence is freed afterwards.

        Counterpart of the reference's rocket-teacher-score
        (engines/glm5-moe-nvfp4-2b/src/teacher_score_main.cu:1-212)."""
        m = self.model
        r = Request(list(map(int, seq)), 1)
        self.kv.open(r.rid, [])
        r.status = Status.PREFILL
        step = max(1, min(self.ecfg.prefill_chunk, m.max_out, m.max_tokens))
        preds: list[int] = []
        try:
            for s0 in range(0, len(seq), step):
                toks = r.prompt[s0:s0 + step]
                sc = ScheduledSeq(r, toks, s0, True)
                T, S, w, _ = self._stage([sc])
                # every row of the chunk is a sampled row
                o = self.meta_off["out_rows"]
                self.meta_host.numpy()[o[0]:o[0] + T] = np.arange(T, dtype=np.int32)
                self.meta_dev.copy_(self.meta_host, non_blocking=True)
                out = m.forward(T, S, w, T, False)
                preds += out[:T].cpu().tolist()
        finally:
            self.kv.free(r.rid)
            sl = self.slot_of.pop(r.rid, None)
            if sl is not None:
                self.free_slots.append(sl)
        return preds

    def teacher_nll(self, seq: list[int]) -> list[float]:
        """Teacher-forced negative log-likelihood (nats) of seq[1:], one value per token:
        -log softmax(logits after seq[:i])[seq[i]].  Eager prefill chunks with every row
        sampled into fp32 logits; under tensor parallelism the log-sum-exp over the
        vocabulary shards and the target logit are combined with two all-reduces.
        Perplexity = exp(mean).  The sequence is freed afterwards."""
        m = self.model
        seq = list(map(int, seq))
        if len(seq) < 2:
            return []
        r = Request(seq, 1)
        self.kv.open(r.rid, [])
        r.status = Status.PREFILL
        step = max(1, min(self.ecfg.prefill_chunk, m.max_out, m.max_tokens, 256))
        buf = torch.empty(step, m.V_l, dtype=torch.float32, device=self.dev)
        n_valid = max(0, min(m.V_l, self.cfg.vocab_size - m.v_lo))
        nll: list[float] = []
        try:
            for s0 in range(0, len(seq) - 1, step):
                toks = seq[s0:s0 + step]
                sc = ScheduledSeq(r, toks, s0, True)
                T, S, w, _ = self._stage([sc])
                o = self.meta_off["out_rows"]
                self.meta_host.numpy()[o[0]:o[0] + T] = np.arange(T, dtype=np.int32)
                self.meta_dev.copy_(self.meta_host, non_blocking=True)
                lg = m.forward(T, S, w, T, False, logits_out=buf)[:T, :n_valid]
                tgt = torch.tensor(seq[s0 + 1:s0 + T + 1], dtype=torch.long, device=self.dev)
                rows = tgt.numel()  # the last chunk's last row predicts past the end
                nll += sharded_token_nll(lg[:rows], tgt, m.v_lo, self.par).cpu().tolist()
        finally:
            self.kv.free(r.rid)
            sl = self.slot_of.pop(r.rid, None)
            if sl is not None:
                self.free_slots.append(sl)
        return nll

    def teacher_logits(self, seq: list[int]) -> torch.Tensor:
        """Teacher-forced fp32 logits [len(seq), V_l] of this rank's vocabulary shard: row i
        is the next-token distribution after seq[:i+1].  The same eager chunks as
        teacher_score / teacher_nll; the sequence is freed afterwards.  Numerics API (the
        multi-GPU parity gates compare these rows across layouts)."""
        m = self.model
        seq = list(map(int, seq))
        r = Request(seq, 1)
        self.kv.open(r.rid, [])
        r.status = Status.PREFILL
        step = max(1, min(self.ecfg.prefill_chunk, m.max_out, m.max_tokens, 256))
        buf = torch.empty(step, m.V_l, dtype=torch.float32, device=self.dev)
        n_valid = max(0, min(m.V_l, self.cfg.vocab_size - m.v_lo))
        rows = []
        try:
            for s0 in range(0, len(seq), step):
                toks = seq[s0:s0 + step]
                sc = ScheduledSeq(r, toks, s0, True)
                T, S, w, _ = self._stage([sc])
                o = self.meta_off["out_rows"]
                self.meta_host.numpy()[o[0]:o[0] + T] = np.arange(T, dtype=np.int32)
                self.meta_dev.copy_(self.meta_host, non_blocking=True)
                rows.append(m.forward(T, S, w, T, False, logits_out=buf)[:T, :n_valid].float().cpu())
        finally:
            self.kv.free(r.rid)
            sl = self.slot_of.pop(r.rid, None)
            if sl is not None:
                self.free_slots.append(sl)
        return torch.cat(rows)

    def spec_summary(self, reqs: list[Request]) -> dict:
        drafted = sum(r.drafted for r in reqs)
        acc = sum(r.accepted for r in reqs)
        out = {"spec_tokens": self.K, "drafted": drafted, "accepted": acc,
               "acceptance": acc / drafted if drafted else None,
               "draft_source": self.drafts.name if self.drafts is not None else "mtp"}
        if self.drafts is not None and hasattr(self.drafts, "hits"):
            out["proposals_by_source"] = dict(self.drafts.hits)
        if self.depth_policy is not None:
            out["depth_policy"] = self.depth_policy.summary()
        return out

    def _sync_decision(self, ids: np.ndarray) -> np.ndarray:
        t = torch.from_numpy(ids).to(self.dev)
        self.par.broadcast(t, 0)
        return t.cpu().numpy()

    def _capture(self, B: int, T: int, W_: int, n_out: int) -> torch.cuda.CUDAGraph:
        """Capture one decode (or speculative verify+draft) step of batch B (metadata staged)."""
        m = self.model
        K = self.K
        if K:
            run = lambda n_verify=B: m.spec_forward(T, B, W_, n_out, T, n_verify, self.dummy_page,
                                                    draft_passes=self._passes())
        else:
            run = lambda n_verify=0: m.forward(T, B, W_, n_out, True)
        torch.cuda.synchronize(self.dev)
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            # warm-up launch outside the graph (lazy workspaces).  It writes KV entries at the
            # slots the replay rewrites.  Recurrent (DeltaNet) state is not idempotent, so the
            # warm-up runs every sequence on the scratch state slot and skips the commit;
            # the real state advances once, in the replay.
            if self.hybrid:
                m.state_slot[:B].fill_(self.dummy_slot)
            run(0)
            if self.hybrid:
                self.meta_dev.copy_(self.meta_host, non_blocking=True)
        torch.cuda.current_stream(self.dev).wait_stream(s)
        torch.cuda.synchronize(self.dev)
        g = torch.cuda.CUDAGraph()
        n0 = ops.launch_count()
        with torch.cuda.graph(g, stream=s):
            run()
        self.kernels_per_decode_step[B] = ops.launch_count() - n0
        torch.cuda.synchronize(self.dev)
        self.graphs[("spec", B, self._width(), self._passes()) if K else B] = g
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
