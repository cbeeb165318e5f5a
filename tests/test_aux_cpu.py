"""Host runtime pieces on the CPU: expert balancing (greedy LPT, equal cardinality,
deterministic) and the Prometheus metrics rendering.

Expert balancing mirrors the reference's expert_balance tests
(engines/glm5-moe-nvfp4-2b/src/fabric/expert_balance.cc:58-102).
"""
import random

from rocket_b200.parallel import expert_balance as eb
from rocket_b200.utils.metrics import Metrics


def test_balance_equal_cardinality_and_better_than_contiguous():
    rnd = random.Random(0)
    E, R = 160, 8
    # skewed: hot experts clustered at low ids (the contiguous split puts them on rank 0)
    hist = [int(1000 * (0.97 ** e) + rnd.randint(0, 20)) for e in range(E)]
    p = eb.placement(hist, R)
    owner, order, load = p["owner"], p["order"], p["rank_load"]
    assert sorted(order) == list(range(E))
    for r in range(R):
        assert sum(1 for o in owner if o == r) == E // R
        assert all(owner[e] == r for e in order[r * E // R:(r + 1) * E // R])
    assert sum(load) == sum(hist)
    contig = eb.contiguous_load(hist, R)
    assert max(load) < max(contig) / 3
    assert max(load) - min(load) <= max(hist)  # LPT bound
    assert eb.balance(hist, R) == order  # deterministic


def test_balance_rejects_bad_shapes():
    import pytest
    with pytest.raises(Exception):
        eb.balance([1, 2, 3], 2)


def test_metrics_render():
    m = Metrics(labels={"rank": 0})
    m.inc("requests_total", 3)
    m.inc("generated_tokens_total", 42)
    m.set("running_requests", 2)
    for v in (3, 7, 40):
        m.observe("step_ms", v)
    txt = m.render()
    assert 'rocket_b200_requests_total{rank="0"} 3' in txt
    assert 'rocket_b200_step_ms_bucket{le="5",rank="0"} 1' in txt
    assert 'rocket_b200_step_ms_count{rank="0"} 3' in txt
    assert "# TYPE rocket_b200_itl_ms histogram" in txt


def test_tracer_bounded_labels_and_exports(tmp_path):
    import json

    import pytest

    from rocket_b200.utils.tracing import NULL_TRACER, Tracer
    tr = Tracer(rank=3, capacity=4)
    with tr.span("step", phase="decode", bucket=64):
        pass
    with pytest.raises(ValueError):
        with tr.span("step", phase="decode"):
            raise ValueError("boom")
    with pytest.raises(ValueError):
        tr.span("step", request_id="r-123")     # unbounded label keys are refused
    for _ in range(5):
        with tr.span("x"):
            pass
    assert len(tr.spans) == 4 and tr.dropped == 3
    tr2 = Tracer(rank=1)
    with tr2.span("a", phase="p"):
        pass
    with pytest.raises(KeyError):
        with tr2.span("a", phase="p"):
            raise KeyError("k")
    outs = [s[1]["outcome"] for s in tr2.spans]
    assert outs == ["ok", "error"] and tr2.spans[0][1]["rank"] == "1"
    assert tr2.summary()["a|p"]["count"] == 2
    tr2.export_chrome(str(tmp_path / "t.json"))
    ev = json.load(open(tmp_path / "t.json"))["traceEvents"]
    assert ev[0]["ph"] == "X" and ev[0]["pid"] == 1
    tr2.export_otlp_json(str(tmp_path / "t.otlp.json"))
    doc = json.load(open(tmp_path / "t.otlp.json"))
    sp = doc["resourceSpans"][0]["scopeSpans"][0]["spans"]
    assert len(sp) == 2 and sp[1]["status"]["code"] == 2 and int(sp[0]["endTimeUnixNano"]) > int(sp[0]["startTimeUnixNano"])
    tr2.export_jsonl(str(tmp_path / "t.jsonl"))
    assert len(open(tmp_path / "t.jsonl").read().splitlines()) == 2
    with NULL_TRACER.span("anything", whatever=1):
        pass


def test_checksum_digest_properties():
    import torch

    from rocket_b200.utils.checksums import digest, first_divergence
    a = torch.arange(1000, dtype=torch.float32)
    assert digest(a) == digest(a.clone())
    b = a.clone()
    b[17] = 17.000002
    assert digest(a) != digest(b)                  # one ulp
    assert digest(a) != digest(a.flip(0))          # permutation
    assert digest(torch.zeros(3, dtype=torch.uint8)) != digest(torch.zeros(5, dtype=torch.uint8))
    s1 = [{"step": 0, "kv": [1, 2]}, {"step": 1, "kv": [3, 4], "spec": 9}]
    s2 = [{"step": 0, "kv": [1, 2]}, {"step": 1, "kv": [3, 5], "spec": 9}]
    assert first_divergence(s1, s1) is None
    assert first_divergence(s1, s2) == (1, "kv")


def test_debug_bounds_build_compiles():
    """The debug bounds-check variant (-DRKT_DEBUG_BOUNDS) of the index-heavy kernels compiles."""
    import os
    import shutil
    import subprocess
    import tempfile

    import pytest
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("no nvcc")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    csrc = os.path.join(root, "rocket_b200", "csrc")
    with tempfile.TemporaryDirectory() as d:
        for f in ("sparse_attn.cu", "mla.cu"):
            r = subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-DRKT_DEBUG_BOUNDS",
                                "-c", os.path.join(csrc, f), "-o", os.path.join(d, f + ".o"), "-I", csrc],
                               capture_output=True, text=True, timeout=600)
            assert r.returncode == 0, r.stderr[-2000:]


def test_every_fuel_loads_and_validates():
    """Every shipped fuel parses, validates (fail-closed schema) and reports its size."""
    import glob
    import os

    from rocket_b200.config import load_fuel
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    names = sorted(os.path.basename(p)[:-5] for p in glob.glob(os.path.join(root, "rocket_b200", "fuels", "*.yaml")))
    assert {"glm-moe-355b", "qwen3-next-hybrid", "glm5-flash-style", "tiny-moe", "tiny-mla"} <= set(names)
    for n in names:
        cfg = load_fuel(n).model
        assert cfg.num_layers > 0 and cfg.d_model % 64 == 0, n


def test_tiny_fuels_run_on_the_cpu_oracle():
    """Each oracle-sized architecture (GQA, DeltaNet, KDA, mHC, DSA, MLA, FP8-row) runs the CPU
    oracle end to end, and the MTP head where the fuel has one."""
    import torch

    from rocket_b200.config import load_fuel
    from rocket_b200.models import ReferenceModel, init_fuel_tensors
    for n in ["tiny-moe", "tiny-hybrid", "tiny-kda", "tiny-hc", "tiny-dsa", "tiny-mla", "tiny-fp8"]:
        cfg = load_fuel(n).model
        t = init_fuel_tensors(cfg, 0)
        ref = ReferenceModel(cfg, t, quantized=True, emulate_gpu=True)
        ids = torch.randint(0, cfg.vocab_size, (24,), generator=torch.Generator().manual_seed(0))
        lg = ref.logits(ids)
        assert lg.shape == (24, cfg.vocab_size) and torch.isfinite(lg).all(), n
        if cfg.mtp_layers:
            _, ml = ref.mtp(ref.hidden_prenorm(ids), ids)
            assert torch.isfinite(ml).all(), n


def test_config_refuses_bad_architecture_fields():
    import dataclasses

    import pytest

    from rocket_b200.config import load_fuel
    from rocket_b200.config.schema import ConfigError, MlaConfig, SparseAttnConfig
    cfg = load_fuel("tiny-moe").model
    for bad in [dict(hc_streams=3), dict(mla=MlaConfig(kv_lora_rank=256)),
                dict(sparse_attention=SparseAttnConfig(index_dim=64)),
                dict(mla=MlaConfig(v_head_dim=128))]:       # head_dim must equal v_head_dim
        with pytest.raises(ConfigError):
            dataclasses.replace(cfg, **bad).validate()


def test_engine_presets_and_overrides():
    import pytest

    from rocket_b200.config.schema import ConfigError, load_engine
    for name in ("glm-bs64-8gpu", "hybrid-mtp", "long-context-fp8"):
        e = load_engine(name)
        assert e.page_size == 64 and e.max_batch in e.batch_buckets
    e = load_engine("long-context-fp8", max_batch=128, kv_dtype=None)
    assert e.max_batch == 128 and e.kv_dtype == "fp8" and e.draft_source == "prompt_lookup+mtp"
    with pytest.raises(ConfigError):
        load_engine("no-such-preset")
    with pytest.raises(ConfigError):
        load_engine({"page_size": 48})
    with pytest.raises(ConfigError):
        load_engine({"not_a_field": 1})
