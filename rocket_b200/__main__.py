"""Command line: ``python -m rocket_b200 <command>``.

  generate   greedy-generate (token ids or text through a tokenizer.json), random-init or
             safetensors weights (--fuel-dir), optional MTP speculation (--spec K)
  score      teacher-forced accuracy and throughput of a fuel on token sequences
  pack-fuel  write a fuel's random-init weights as a safetensors checkpoint (small fuels)
  serve-bench  open-loop serving benchmark: Poisson arrivals, uniform prompt lengths,
             geometric outputs (the long-context sweep's shape; torchrun-aware)
  static-fire  parity gate: `--mode single` writes reference tokens on one GPU, `--mode
             parallel` (under torchrun) regenerates them with N ranks and counts mismatches
  agent-trace  forked-prefix agent workload trace (JSONL) with its KV-sharing summary;
             `--validate --trace FILE` checks causality (serve-bench / http-bench replay it)
  http-bench   load generator against an OpenAI-style completions server (Poisson or
             agent-trace replay; streaming, client-side TTFT / ITL)
  quality    deterministic task set + long-context needles against a completions server;
             `--compare base.json` exits 1 on regressions
  perplexity teacher-forced perplexity of a text (tokenizer) or a token-id file
  stages     per-stage GPU time of one decode step (stage timer)
  probe      mount probe: device facts + a trivial kernel (the reference's test stand)

Counterparts of the reference's rocket-decode / rocket-teacher-score / rocket-test-stand
binaries (engines/glm5-moe-nvfp4-2b/src/decode_main.cu, teacher_score_main.cu, test_stand.cu).
"""
from __future__ import annotations

import argparse
import json
import sys


def _agent_args(p):
    g = p.add_argument_group("agent workload")
    g.add_argument("--concurrency", type=int, default=16, help="sessions served per tick")
    g.add_argument("--depth", type=int, default=2, help="fork depth limit")
    g.add_argument("--prefix-tokens", type=int, default=8192, help="shared root prefix")
    g.add_argument("--tool-burst-tokens", type=int, default=300)
    g.add_argument("--duration-steps", type=int, default=2000, help="ticks")
    g.add_argument("--seed", type=int, default=0)
    g.add_argument("--max-context", type=int, default=None, help="end sessions past this context")


def _agent_events(a):
    from .engine.agent_workload import agent_trace, read_trace
    if a.trace:
        return [e for e in read_trace(a.trace) if e.get("event") != "summary"]
    return agent_trace(a.concurrency, a.depth, a.prefix_tokens, a.tool_burst_tokens, a.duration_steps, a.seed,
                       max_context=a.max_context)


def main(argv=None):
    ap = argparse.ArgumentParser(prog="rocket_b200")
    sub = ap.add_subparsers(dest="cmd", required=True)
    g = sub.add_parser("generate")
    g.add_argument("--fuel", default="glm-moe-small")
    g.add_argument("--fuel-dir", default=None, help="safetensors checkpoint directory (default: random init)")
    g.add_argument("--prompt", type=str, default="1,2,3,4", help="comma-separated token ids")
    g.add_argument("--text", type=str, default=None, help="prompt text (needs --tokenizer)")
    g.add_argument("--tokenizer", default=None, help="tokenizer.json")
    g.add_argument("--max-new-tokens", type=int, default=16)
    g.add_argument("--spec", type=int, default=0, help="MTP draft tokens per step")
    g.add_argument("--draft-source", default="mtp",
                   help="'+'-joined priority list: mtp | prompt_lookup | history | file")
    g.add_argument("--draft-file", default=None, help="reference generation (JSON) for --draft-source file")
    g.add_argument("--draft-fuel", default=None, help="draft model fuel for --draft-source draft_model")
    g.add_argument("--draft-fuel-dir", default=None, help="draft model checkpoint (default: random init)")
    g.add_argument("--prompt-file", default=None, help="prompt as a text file (needs --tokenizer) or a JSON id list")
    g.add_argument("--prompt-list", default=None, help="JSON lines, one prompt (text or id list) each: a batch")
    g.add_argument("--batch", type=int, default=1, help="run every prompt this many times concurrently")
    g.add_argument("--kv-pages", type=int, default=None, help="KV pages (default: from free memory)")
    g.add_argument("--no-cuda-graph", action="store_true")
    g.add_argument("--prefix-cache-dir", default=None, help="persistent prefix tier (NVMe) under this directory")
    g.add_argument("--prefix-cache-gib", type=int, default=64)
    g.add_argument("--telemetry", action="store_true", help="print layer RMS / router entropy of the prompt")
    g.add_argument("--expert-cache-slots", type=int, default=0,
                   help="stream routed experts from host memory into this many device slots per layer")
    g.add_argument("--result-json", default=None)
    sc = sub.add_parser("score")
    sc.add_argument("--fuel", default="glm-moe-small")
    sc.add_argument("--fuel-dir", default=None)
    sc.add_argument("--seqs", type=int, default=4)
    sc.add_argument("--len", type=int, default=256)
    sc.add_argument("--ids-file", default=None, help="JSON list of token-id lists (default: random ids)")
    pf = sub.add_parser("pack-fuel")
    pf.add_argument("--fuel", default="tiny-moe")
    pf.add_argument("--out", required=True)
    pf.add_argument("--seed", type=int, default=0)
    pf.add_argument("--shard-mib", type=int, default=4096)
    qf = sub.add_parser("quantize-fuel", help="bf16/fp32 safetensors checkpoint -> NVFP4 fuel directory")
    qf.add_argument("--src", required=True, help="checkpoint directory or .safetensors file")
    qf.add_argument("--out", required=True)
    qf.add_argument("--fuel", default="glm-moe-355b", help="fuel whose weight_format decides what is NVFP4")
    qf.add_argument("--shard-mib", type=int, default=4096)
    qf.add_argument("--threads", type=int, default=0)
    ps = sub.add_parser("pack-slabs", help="write per-EP-rank expert slabs (64 KiB-aligned slots)")
    ps.add_argument("--fuel", default="tiny-moe")
    ps.add_argument("--fuel-dir", required=True)
    ps.add_argument("--out", required=True)
    ps.add_argument("--world", type=int, default=8)
    vf = sub.add_parser("verify-fuel", help="check every shard against checksums.txt")
    vf.add_argument("--dir", required=True)
    sv = sub.add_parser("serve", help="OpenAI-style HTTP completions server (rank 0 serves; others follow)")
    sv.add_argument("--fuel", default="glm-moe-small")
    sv.add_argument("--fuel-dir", default=None)
    sv.add_argument("--tokenizer", default=None, help="tokenizer.json for text prompts / outputs")
    sv.add_argument("--host", default="127.0.0.1")
    sv.add_argument("--port", type=int, default=8000)
    sv.add_argument("--api-key", default=None)
    sv.add_argument("--max-queue", type=int, default=None,
                    help="requests waiting for admission beyond this get HTTP 429 (default: unbounded)")
    sv.add_argument("--chat-template", default=None,
                    help="Jinja chat template file (default: the tokenizer_config.json beside --tokenizer)")
    sv.add_argument("--engine-config", default=None,
                    help="engine YAML or preset name (rocket_b200/engines); flags below override it")
    sv.add_argument("--max-batch", type=int, default=None)
    sv.add_argument("--max-seq-len", type=int, default=None)
    sv.add_argument("--chunk", type=int, default=None)
    sv.add_argument("--spec", type=int, default=None)
    sv.add_argument("--draft-source", default=None)
    sv.add_argument("--kv-dtype", default=None, choices=["bf16", "fp8"])
    sv.add_argument("--expert-cache-slots", type=int, default=None,
                    help="stream routed experts from host memory into this many device slots per layer")
    rt = sub.add_parser("route", help="one HTTP endpoint over several serve backends (data parallel)")
    rt.add_argument("--backend", action="append", required=True, help="backend base URL (repeat)")
    rt.add_argument("--host", default="127.0.0.1")
    rt.add_argument("--port", type=int, default=8000)
    rt.add_argument("--api-key", default=None)
    sb = sub.add_parser("serve-bench")
    sb.add_argument("--fuel", default="glm-moe-355b")
    sb.add_argument("--requests", type=int, default=64)
    sb.add_argument("--rate", type=float, default=0.0, help="requests/s (0 = all arrive at once, saturating)")
    sb.add_argument("--prompt-lo", type=int, default=1024)
    sb.add_argument("--prompt-hi", type=int, default=8192)
    sb.add_argument("--mean-out", type=float, default=512)
    sb.add_argument("--max-out", type=int, default=2048)
    sb.add_argument("--max-batch", type=int, default=64)
    sb.add_argument("--chunk", type=int, default=8192)
    sb.add_argument("--spec", type=int, default=0)
    sb.add_argument("--draft-source", default="mtp")
    sb.add_argument("--kv-dtype", default="bf16", choices=["bf16", "fp8"])
    sb.add_argument("--time-limit", type=float, default=None)
    sb.add_argument("--workload", choices=["poisson", "agent"], default="poisson",
                    help="agent: replay a forked-prefix agent trace (--trace, or generated from the agent flags)")
    sb.add_argument("--trace", default=None, help="agent trace JSONL (python -m rocket_b200 agent-trace)")
    _agent_args(sb)
    fh = sub.add_parser("fuel-from-hf", help="fuel YAML from a Hugging Face config.json (glm4_moe, qwen3_next, "
                                             "qwen3_moe)")
    fh.add_argument("--config", required=True)
    fh.add_argument("--id", default=None, help="fuel id (default: the config's model_type)")
    fh.add_argument("--out", default=None)
    ih = sub.add_parser("import-hf", help="Hugging Face checkpoint dir -> fuel dir (renamed, re-laid-out tensors, "
                                          "fuel.yaml)")
    ih.add_argument("--src", required=True)
    ih.add_argument("--out", required=True)
    ih.add_argument("--id", default=None)
    qg = sub.add_parser("quality", help="deterministic task set + needles against a completions server")
    qg.add_argument("--url", required=True)
    qg.add_argument("--model", default=None)
    qg.add_argument("--max-tokens", type=int, default=1024)
    qg.add_argument("--needles", default="8000,64000", help="comma-separated needle depths in tokens")
    qg.add_argument("--timeout", type=float, default=900.0)
    qg.add_argument("--out", required=True)
    qg.add_argument("--compare", default=None, help="baseline report: exit 1 on any regression")
    pp = sub.add_parser("perplexity", help="teacher-forced perplexity of a text or token-id file")
    pp.add_argument("--fuel", default="glm-moe-small")
    pp.add_argument("--fuel-dir", default=None)
    pp.add_argument("--tokenizer", default=None)
    pp.add_argument("--text-file", default=None)
    pp.add_argument("--ids-file", default=None, help="JSON list of token ids")
    pp.add_argument("--window", type=int, default=2048)
    pp.add_argument("--stride", type=int, default=None)
    pp.add_argument("--max-tokens", type=int, default=None, help="score at most this many tokens")
    at = sub.add_parser("agent-trace", help="write / validate a forked-prefix agent workload trace (JSONL)")
    _agent_args(at)
    at.add_argument("--fuel", default="glm-moe-355b", help="model whose KV cost the summary uses")
    at.add_argument("--kv-dtype", default="bf16", choices=["bf16", "fp8"])
    at.add_argument("--out", default=None, help="output file (default stdout)")
    at.add_argument("--validate", action="store_true", help="check the causality of --trace and exit")
    at.add_argument("--trace", default=None)
    hb = sub.add_parser("http-bench", help="load generator against an OpenAI-style completions server")
    hb.add_argument("--url", required=True)
    hb.add_argument("--model", default=None)
    hb.add_argument("--api-key", default=None)
    hb.add_argument("--workload", choices=["poisson", "agent"], default="poisson")
    hb.add_argument("--trace", default=None)
    hb.add_argument("--vocab", type=int, default=151552, help="token ids are drawn from [0, vocab)")
    hb.add_argument("--requests", type=int, default=64)
    hb.add_argument("--rate", type=float, default=0.0)
    hb.add_argument("--prompt-lo", type=int, default=1024)
    hb.add_argument("--prompt-hi", type=int, default=8192)
    hb.add_argument("--mean-out", type=float, default=256)
    hb.add_argument("--max-out", type=int, default=2048)
    hb.add_argument("--max-inflight", type=int, default=64)
    hb.add_argument("--time-limit", type=float, default=None)
    _agent_args(hb)
    sf = sub.add_parser("static-fire")
    sf.add_argument("--fuel", default="glm-moe-small")
    sf.add_argument("--mode", choices=["single", "parallel"], required=True)
    sf.add_argument("--ref", required=True, help="reference token file (written in single mode)")
    sf.add_argument("--prompts", type=int, default=8)
    sf.add_argument("--len", type=int, default=128)
    sf.add_argument("--tokens", type=int, default=16)
    sf.add_argument("--max-mismatch", type=int, default=0)
    sf.add_argument("--layout", choices=["exact", "tp"], default="exact",
                    help="exact: attention replicated (TP=1), experts EP=N -- the step must reproduce one GPU "
                         "bit for bit; tp: TP=N attention / dense / vocab + EP=N experts")
    sf.add_argument("--collectives", choices=["fused", "sp", "nccl"], default="fused")
    sf.add_argument("--fuel-dir", default=None, help="checkpoint directory (default: seeded random fuel tensors)")
    s = sub.add_parser("stages")
    s.add_argument("--fuel", default="glm-moe-355b")
    s.add_argument("--batch", type=int, default=64)
    s.add_argument("--ctx", type=int, default=2048)
    s.add_argument("--splits", type=int, default=1)
    s.add_argument("--graph", action="store_true", help="time the step inside a captured CUDA graph")
    s.add_argument("--kernels", action="store_true", help="per-kernel device time of graph replays (CUPTI)")
    sub.add_parser("probe")
    a = ap.parse_args(argv)

    import torch

    from .config import EngineConfig, load_fuel
    from .engine import LLMEngine

    if a.cmd == "probe":
        from .utils.probe import probe_mount
        print(json.dumps(probe_mount(), indent=1))
        return
    if a.cmd == "pack-fuel":
        from .fuel.safetensors_io import save_dir
        from .models import init_fuel_tensors
        cfg = load_fuel(a.fuel).model
        t = {k: v for k, v in init_fuel_tensors(cfg, a.seed).items() if not k.startswith("master.")}
        save_dir(t, a.out, shard_bytes=a.shard_mib << 20, meta={"fuel": a.fuel, "seed": str(a.seed)})
        print(json.dumps({"fuel": a.fuel, "out": a.out, "tensors": len(t),
                          "bytes": sum(v.numel() * v.element_size() for v in t.values())}))
        return
    if a.cmd == "route":
        import uvicorn

        from .serve_router import backends_from_urls, build_router
        uvicorn.run(build_router(backends_from_urls(a.backend), api_key=a.api_key), host=a.host, port=a.port,
                    log_level="warning")
        return
    if a.cmd == "serve":
        from .parallel import init_from_env
        from .serve import EngineLoop, build_app, follow
        from .config.schema import load_engine
        par = init_from_env(timeout_s=3600)
        base = a.engine_config or {"max_batch": 64, "max_seq_len": 8192, "prefill_chunk": 8192}
        ecfg = load_engine(base, tp=par.world, ep=par.world, max_batch=a.max_batch, prefill_chunk=a.chunk,
                           max_seq_len=a.max_seq_len, spec_tokens=a.spec, draft_source=a.draft_source,
                           kv_dtype=a.kv_dtype, expert_cache_slots=a.expert_cache_slots)
        eng = LLMEngine.from_fuel(a.fuel, ecfg, par=par, fuel_dir=a.fuel_dir)
        if par.rank != 0:
            follow(eng)
            return
        tok, tpl, eos = None, None, []
        if a.tokenizer:
            from .fuel.tokenizer import Tokenizer
            from .serve import chat_config
            tok = Tokenizer.from_file(a.tokenizer)
            tpl, eos_strs = chat_config(a.tokenizer)
            eos = [i for e in eos_strs for i in tok.encode(e, allow_special=True)[-1:]]
        if a.chat_template:
            with open(a.chat_template) as f:
                tpl = f.read()
        import uvicorn
        loop = EngineLoop(eng, par, max_pending=a.max_queue).start()
        try:
            uvicorn.run(build_app(loop, a.fuel, tok, a.api_key, chat_template=tpl, eos_ids=eos), host=a.host,
                        port=a.port, log_level="warning")
        finally:
            loop.stop()
            eng.release_graphs()
        return
    if a.cmd == "quantize-fuel":
        from .fuel.materialize import materialize
        rep = materialize(a.src, a.out, load_fuel(a.fuel).model.weight_format, a.shard_mib << 20, a.threads,
                          meta={"fuel": a.fuel})
        print(json.dumps(rep))
        return
    if a.cmd == "pack-slabs":
        from .fuel.safetensors_io import load_dir
        from .fuel.slabs import pack_expert_slabs
        paths = pack_expert_slabs(load_dir(a.fuel_dir), load_fuel(a.fuel).model, a.out, a.world, fuel=a.fuel)
        print(json.dumps({"slabs": paths}))
        return
    if a.cmd == "verify-fuel":
        from .fuel.materialize import verify
        bad = verify(a.dir)
        print(json.dumps({"dir": a.dir, "bad_shards": bad}))
        sys.exit(1 if bad else 0)
    if a.cmd == "generate":
        import time
        tok = None
        if a.tokenizer:
            from .fuel.tokenizer import Tokenizer
            tok = Tokenizer.from_file(a.tokenizer)

        def as_ids(p):
            if isinstance(p, list):
                return [int(x) for x in p]
            if tok is None:
                raise SystemExit("text prompts need --tokenizer")
            return tok.encode(p)
        if a.prompt_list:  # JSON lines: one prompt (text or a list of ids) per line
            with open(a.prompt_list) as f:
                prompts = [as_ids(json.loads(ln)) for ln in f if ln.strip()]
        elif a.prompt_file:  # a text file, or a JSON list of token ids
            with open(a.prompt_file) as f:
                raw = f.read()
            try:
                js = json.loads(raw)
            except ValueError:
                js = raw
            prompts = [as_ids(js)]
        elif a.text is not None:
            prompts = [as_ids(a.text)]
        else:
            prompts = [[int(x) for x in a.prompt.split(",")]]
        if a.batch > 1:
            prompts = [p for p in prompts for _ in range(a.batch)]
        B = len(prompts)
        buckets = sorted({1, 2, 4, 8, 16, 32, 64, 128, 256} | {B})
        longest = max(len(p) for p in prompts)
        ecfg = EngineConfig(max_batch=max(4, B), prefill_chunk=max(2048, min(8192, longest)),
                            max_seq_len=max(4096, longest + a.max_new_tokens + 64),
                            batch_buckets=[b for b in buckets if b <= max(4, B)], spec_tokens=a.spec,
                            draft_source=a.draft_source, draft_file=a.draft_file or "",
                            expert_cache_slots=a.expert_cache_slots, cuda_graphs=not a.no_cuda_graph,
                            prefix_cache=True)
        # default KV: room for every request's prompt + output (+ speculative slack) and some spare pages
        kv_pages = a.kv_pages or B * -(-(longest + a.max_new_tokens + 2 * a.spec + 64) // 64) + 16
        a.kv_pages = kv_pages
        draft = None
        if "draft_model" in a.draft_source.split("+"):
            if not a.draft_fuel:
                raise SystemExit("--draft-source draft_model needs --draft-fuel")
            ecfg.draft_source = "history"  # placeholder until the draft engine is attached
            draft = LLMEngine.from_fuel(a.draft_fuel, EngineConfig(max_batch=ecfg.max_batch, prefill_chunk=2048,
                                                                   max_seq_len=ecfg.max_seq_len,
                                                                   batch_buckets=ecfg.batch_buckets),
                                        fuel_dir=a.draft_fuel_dir, kv_pages=a.kv_pages)
        eng = LLMEngine.from_fuel(a.fuel, ecfg, kv_pages=a.kv_pages, fuel_dir=a.fuel_dir)
        if draft is not None:
            eng.set_draft_source(a.draft_source, a.draft_file, draft_engine=draft)
        if a.prefix_cache_dir:
            from .kv.prefix_store import PrefixTier
            eng.attach_prefix_tier(PrefixTier(eng, a.prefix_cache_dir, max_bytes=a.prefix_cache_gib << 30))
        res = {}
        if a.telemetry:
            from .utils.telemetry import Telemetry
            tel = Telemetry(eng.model)
            with tel:
                eng.prompt_logits(prompts[0])
            res["telemetry"] = tel.summary()
        t0 = time.perf_counter()
        reqs = [eng.add_request(p, a.max_new_tokens) for p in prompts]
        while eng.sched.has_work():
            eng.step()
        dt = time.perf_counter() - t0
        n_out = sum(len(r.output) for r in reqs)
        res.update({"requests": B, "prompt_tokens": sum(len(p) for p in prompts), "seconds": round(dt, 4),
                    "tok_s": round(n_out / dt, 2), **LLMEngine.latency_summary(reqs)})
        if B == 1:
            res["output"] = reqs[0].output
        else:
            res["outputs"] = [r.output for r in reqs]
        if a.spec:
            res["spec"] = eng.spec_summary(reqs)
        if tok is not None:
            if B == 1:
                res["text"] = tok.decode(reqs[0].output)
            else:
                res["texts"] = [tok.decode(r.output) for r in reqs]
        print(json.dumps(res))
        if a.result_json:
            with open(a.result_json, "w") as f:
                json.dump(res, f, indent=1)
        return
    if a.cmd == "score":
        import time
        cfg = load_fuel(a.fuel).model
        if a.ids_file:
            with open(a.ids_file) as f:
                seqs = json.load(f)
        else:
            g = torch.Generator().manual_seed(0)
            seqs = [torch.randint(0, cfg.vocab_size, (a.len,), generator=g).tolist() for _ in range(a.seqs)]
        L = max(len(x) for x in seqs)
        ecfg = EngineConfig(max_batch=64, prefill_chunk=max(512, L), max_seq_len=L + 64, cuda_graphs=False,
                            prefix_cache=False)
        eng = LLMEngine.from_fuel(a.fuel, ecfg, kv_pages=(L // 64 + 2) * 2 + 2, fuel_dir=a.fuel_dir)
        hit = tot = 0
        t0 = time.perf_counter()
        for sq in seqs:
            pred = eng.teacher_score(sq)
            hit += sum(int(p == t) for p, t in zip(pred[:-1], sq[1:]))
            tot += len(sq) - 1
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        print(json.dumps({"fuel": a.fuel, "sequences": len(seqs), "positions": tot,
                          "accuracy": round(hit / max(tot, 1), 4), "tok_s": round(sum(map(len, seqs)) / dt, 1)}))
        return
    if a.cmd == "static-fire":
        # counterpart of the reference's static fire (engines/glm5-moe-nvfp4-2b/src/fabric/static_fire.cu)
        from .parallel import init_from_env
        par = init_from_env(timeout_s=300)
        cfg = load_fuel(a.fuel).model
        g = torch.Generator().manual_seed(0)
        prompts = [torch.randint(0, cfg.vocab_size, (a.len,), generator=g).tolist() for _ in range(a.prompts)]
        tp = 1 if a.layout == "exact" else par.world
        ecfg = EngineConfig(tp=tp, ep=par.world, max_batch=a.prompts, prefill_chunk=max(2048, a.len),
                            max_seq_len=a.len + a.tokens + 64, batch_buckets=[a.prompts], prefix_cache=False,
                            collectives=a.collectives)
        tensors = None
        if a.fuel_dir is None:
            # the same seeded fuel tensors on one GPU and on N (sharded at load)
            from .models import init_fuel_tensors
            tensors = init_fuel_tensors(cfg, 0)
        eng = LLMEngine.from_fuel(a.fuel, ecfg, par=par, kv_pages=a.prompts * ((a.len + a.tokens) // 64 + 2) + 2,
                                  tensors=tensors, fuel_dir=a.fuel_dir)
        outs = eng.generate(prompts, max_new_tokens=a.tokens)
        eng.release_graphs()
        if a.mode == "single":
            if par.world != 1:
                raise SystemExit("single mode runs on one GPU")
            with open(a.ref, "w") as f:
                json.dump({"fuel": a.fuel, "outputs": outs}, f)
            print(json.dumps({"mode": "single", "written": a.ref, "sequences": len(outs)}))
            return
        with open(a.ref) as f:
            ref = json.load(f)["outputs"]
        mism = sum(int(x != y) for o, rr in zip(outs, ref) for x, y in zip(o, rr))
        first = [next((i for i, (x, y) in enumerate(zip(o, rr)) if x != y), None) for o, rr in zip(outs, ref)]
        if par.rank == 0:
            print(json.dumps({"mode": "parallel", "n_gpus": par.world, "layout": a.layout,
                              "collectives": a.collectives, "mismatched_tokens": mism,
                              "total_tokens": sum(map(len, outs)), "first_mismatch": first,
                              "pass": mism <= a.max_mismatch}))
        if par.world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
        if mism > a.max_mismatch:
            sys.exit(1)
        return
    if a.cmd == "serve-bench":
        from .engine.loadgen import poisson_workload, run_open_loop
        from .parallel import init_from_env
        par = init_from_env(timeout_s=600)
        cfg = load_fuel(a.fuel).model
        max_seq = a.prompt_hi + a.max_out + 64
        ecfg = EngineConfig(tp=par.world, ep=par.world, max_batch=a.max_batch, prefill_chunk=a.chunk,
                            max_seq_len=max_seq, batch_buckets=sorted({1, 2, 4, 8, 16, 32, 64, 128, 256, a.max_batch}),
                            prefix_cache=False, spec_tokens=a.spec, kv_dtype=a.kv_dtype,
                            draft_source=a.draft_source)
        if a.workload == "agent":
            from .engine.agent_workload import EngineBackend, replay_trace
            max_seq = a.max_context or max_seq
            if a.max_context is None:
                a.max_context = max_seq - 64
            ecfg.max_seq_len, ecfg.prefix_cache = max_seq, True
            eng = LLMEngine.from_fuel(a.fuel, ecfg, par=par)
            res = replay_trace(EngineBackend(eng), _agent_events(a), cfg.vocab_size, seed=a.seed,
                               time_limit_s=a.time_limit)
            eng.release_graphs()
            if par.rank == 0:
                res.update({"fuel": a.fuel, "n_gpus": par.world, "workload": "agent", "concurrency": a.concurrency,
                            "prefix_tokens": a.prefix_tokens, "spec": a.spec})
                print(json.dumps(res), flush=True)
            return
        eng = LLMEngine.from_fuel(a.fuel, ecfg, par=par)
        wl = poisson_workload(a.requests, a.rate or None, (a.prompt_lo, a.prompt_hi), a.mean_out, cfg.vocab_size,
                              max_out=a.max_out)
        res = run_open_loop(eng, wl, a.time_limit)
        eng.release_graphs()
        if par.rank == 0:
            res.update({"fuel": a.fuel, "n_gpus": par.world, "kv_dtype": a.kv_dtype, "spec": a.spec,
                        "prompt": [a.prompt_lo, a.prompt_hi], "mean_out": a.mean_out, "rate": a.rate or "saturate"})
            print(json.dumps(res), flush=True)
        return
    if a.cmd == "fuel-from-hf":
        from .config.hf import fuel_yaml_from_hf
        with open(a.config) as f:
            hf = json.load(f)
        doc = fuel_yaml_from_hf(hf, a.id or hf.get("model_type", "fuel"))
        if a.out:
            with open(a.out, "w") as f:
                f.write(doc)
        else:
            print(doc)
        return
    if a.cmd == "import-hf":
        from .fuel.hf_import import import_hf
        print(json.dumps(import_hf(a.src, a.out, a.id)))
        return
    if a.cmd == "quality":
        from .quality import regressions, run_quality, write_report
        needles = [int(x) for x in a.needles.split(",") if x.strip()]
        rep = run_quality(a.url, a.max_tokens, needles, a.model, a.timeout)
        for name, r in rep["results"].items():
            print(f"{name}\t{'PASS' if r['ok'] else 'FAIL'}\t{r['seconds']}s", flush=True)
        print(f"score\t{rep['passed']}/{rep['total']}")
        write_report(rep, a.out)
        if a.compare:
            with open(a.compare) as f:
                reg = regressions(rep, json.load(f))
            print("regressions\t" + (",".join(reg) or "none"))
            if reg:
                sys.exit(1)
        return
    if a.cmd == "perplexity":
        from .parallel import init_from_env
        from .quality import perplexity
        if a.ids_file:
            with open(a.ids_file) as f:
                ids = [int(x) for x in json.load(f)]
        elif a.text_file and a.tokenizer:
            from .fuel.tokenizer import Tokenizer
            with open(a.text_file, encoding="utf-8") as f:
                ids = Tokenizer.from_file(a.tokenizer).encode(f.read())
        else:
            sys.exit("perplexity needs --ids-file, or --text-file with --tokenizer")
        if a.max_tokens:
            ids = ids[:a.max_tokens]
        par = init_from_env(timeout_s=600)
        # teacher-forced chunks sample every row: the sampled-row limit (max_batch) sets the chunk
        ecfg = EngineConfig(tp=par.world, ep=par.world, max_batch=64, prefill_chunk=256,
                            max_seq_len=a.window + 64, batch_buckets=[1], cuda_graphs=False, prefix_cache=False)
        eng = LLMEngine.from_fuel(a.fuel, ecfg, par=par, fuel_dir=a.fuel_dir, kv_pages=a.window // 64 + 8)
        res = perplexity(eng, ids, a.window, a.stride)
        if par.rank == 0:
            res.update({"fuel": a.fuel, "weights": a.fuel_dir or "random-init", "n_gpus": par.world})
            print(json.dumps(res), flush=True)
        return
    if a.cmd == "agent-trace":
        from .engine.agent_workload import kv_costs, read_trace, trace_summary, validate_trace, write_trace
        if a.validate:
            if not a.trace:
                sys.exit("--validate needs --trace")
            errs = validate_trace(read_trace(a.trace))
            for e in errs[:50]:
                print(e, file=sys.stderr)
            print(json.dumps({"valid": not errs, "errors": len(errs)}))
            sys.exit(1 if errs else 0)
        ev = _agent_events(a)
        per_tok, fixed = kv_costs(load_fuel(a.fuel).model, a.kv_dtype)
        write_trace(ev, a.out or sys.stdout, trace_summary(ev, per_tok, fixed))
        return
    if a.cmd == "http-bench":
        from .serve_client import HttpBackend, run_http_open_loop
        if a.workload == "agent":
            from .engine.agent_workload import replay_trace
            be = HttpBackend(a.url, a.max_inflight, a.model, a.api_key)
            try:
                res = replay_trace(be, _agent_events(a), a.vocab, seed=a.seed, time_limit_s=a.time_limit)
            finally:
                be.close()
        else:
            from .engine.loadgen import poisson_workload
            wl = poisson_workload(a.requests, a.rate or None, (a.prompt_lo, a.prompt_hi), a.mean_out, a.vocab,
                                  max_out=a.max_out)
            res = run_http_open_loop(a.url, wl, a.max_inflight, a.model, a.api_key)
        res.update({"url": a.url, "workload": a.workload})
        print(json.dumps(res), flush=True)
        return
    if a.cmd == "stages":
        from .engine.profile import profile_decode
        from .parallel import init_from_env
        par = init_from_env()
        cfg = load_fuel(a.fuel).model
        max_seq = a.ctx + 64
        ecfg = EngineConfig(tp=par.world, ep=par.world, max_batch=a.batch, prefill_chunk=max(256, a.batch),
                            max_seq_len=max_seq, cuda_graphs=False, prefix_cache=False, batch_buckets=[a.batch])
        pages = a.batch * (-(-max_seq // 64)) + 2
        eng = LLMEngine.from_fuel(a.fuel, ecfg, par=par, kv_pages=pages)
        if a.splits > 1:
            eng.model.set_decode_splits(a.splits, a.batch)
        if a.kernels:
            from .engine.profile import profile_decode_kernels
            res = profile_decode_kernels(eng, a.batch, a.ctx)
            if par.rank == 0:
                print(json.dumps(res, indent=1))
            return
        res = profile_decode(eng, a.batch, a.ctx, graph=a.graph)
        if par.rank != 0:
            return
        tot = sum(v for k, v in res.items() if not k.startswith("_"))
        rows = sorted(((k, v) for k, v in res.items() if not k.startswith("_")), key=lambda kv: -kv[1])
        print(json.dumps({"fuel": a.fuel, "batch": a.batch, "ctx": a.ctx, "step_ms": res.get("_step_ms"),
                          "host_ms": res.get("_host_ms"), "stages_sum_ms": tot,
                          "stages": {k: round(v, 3) for k, v in rows}}, indent=1))


if __name__ == "__main__":
    main()
