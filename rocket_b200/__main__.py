"""Command line: ``python -m rocket_b200 <command>``.

  generate  greedy-generate from prompts (token ids) with a fuel's random-init weights
  stages    per-stage GPU time of one decode step (stage timer)
  probe     mount probe: device facts + a trivial kernel (the reference's test stand)
"""
from __future__ import annotations

import argparse
import json
import sys


def main(argv=None):
    ap = argparse.ArgumentParser(prog="rocket_b200")
    sub = ap.add_subparsers(dest="cmd", required=True)
    g = sub.add_parser("generate")
    g.add_argument("--fuel", default="glm-moe-small")
    g.add_argument("--prompt", type=str, default="1,2,3,4")
    g.add_argument("--max-new-tokens", type=int, default=16)
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
    if a.cmd == "generate":
        ecfg = EngineConfig(max_batch=4, prefill_chunk=2048, max_seq_len=4096, batch_buckets=[1, 2, 4])
        eng = LLMEngine.from_fuel(a.fuel, ecfg, kv_pages=256)
        ids = [int(x) for x in a.prompt.split(",")]
        print(json.dumps({"output": eng.generate([ids], a.max_new_tokens)[0]}))
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
