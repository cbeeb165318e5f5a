"""GPU checks of the auxiliary subsystems: bounded device waits (failure detection
without a fault), telemetry, expert placement, safetensors fuel loading, teacher
scoring, the persistent prefix tier and session checkpoint / resume."""
import os

import pytest
import torch

from rocket_b200 import ops
from rocket_b200.config import EngineConfig, load_fuel
from rocket_b200.engine import LLMEngine
from rocket_b200.models import init_fuel_tensors

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny():
    cfg = load_fuel("tiny-moe").model
    return cfg, init_fuel_tensors(cfg, 0)


def _engine(cfg, t, name="tiny-moe", **kw):
    e = EngineConfig(max_batch=4, batch_buckets=[4], prefill_chunk=512, max_seq_len=320,
                     cuda_graphs=kw.pop("graphs", True), prefix_cache=kw.pop("prefix", False),
                     spec_tokens=kw.pop("spec", 0))
    return LLMEngine.from_fuel(name, e, tensors=kw.pop("tensors", t), kv_pages=kw.pop("pages", 64), cfg_override=cfg,
                               **kw)


def _prompts(cfg, n=2, L=100, seed=11):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, cfg.vocab_size, (L,), generator=g).tolist() for _ in range(n)]


def test_bounded_flag_wait_times_out_and_context_survives():
    dev = torch.device("cuda")
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.ext().flag_wait(flag, 1, 50_000, err)  # nothing ever sets the flag: 50 ms budget
    torch.cuda.synchronize()
    assert int(err.item()) & 2  # kErrPeerTimeout
    err.zero_()
    flag.fill_(1)
    ops.ext().flag_wait(flag, 1, 50_000, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert float((torch.ones(8, device=dev) * 2).sum()) == 16.0  # the context is still usable


def test_telemetry_and_expert_order(tiny):
    from rocket_b200.utils.telemetry import Telemetry
    cfg, t = tiny
    p = _prompts(cfg, 1)[0]
    eng = _engine(cfg, t, graphs=False)
    with Telemetry(eng.model) as tel:
        base = eng.prompt_logits(p)
    s = tel.summary()
    assert len(s["layer_rms"]) == cfg.num_layers and all(v > 0 for v in s["layer_rms"].values())
    assert all(0 < v <= 1.0 for v in s["router_entropy"].values())
    moe_layers = sum(1 for i in range(cfg.num_layers) if cfg.is_moe_layer(i))
    assert s["expert_fires"] == len(p) * cfg.top_k * moe_layers
    hist = tel.fire_histogram()
    assert int(hist.sum()) == s["expert_fires"]
    from rocket_b200.parallel.expert_balance import balance
    order = balance(hist.tolist(), 2)
    assert sorted(order) == list(range(cfg.num_experts))
    perm = _engine(cfg, t, graphs=False, expert_order=order[::-1])
    got = perm.prompt_logits(p)
    cos = torch.nn.functional.cosine_similarity(got, base, 0).item()
    assert cos > 0.999, cos


def test_fuel_dir_and_teacher_score(tiny, tmp_path):
    from rocket_b200.fuel.safetensors_io import load_dir, save_dir
    cfg, t = tiny
    save_dir({k: v for k, v in t.items() if not k.startswith("master.")}, str(tmp_path), shard_bytes=4 << 20)
    p = _prompts(cfg, 1)[0]
    a = _engine(cfg, t, graphs=False).prompt_logits(p)
    b = _engine(cfg, None, graphs=False, tensors=load_dir(str(tmp_path))).prompt_logits(p)
    assert torch.equal(a, b)
    eng = _engine(cfg, t, graphs=False)
    preds = eng.teacher_score(p[:40])
    assert len(preds) == 40
    for i in (9, 25, 39):
        lg = eng.prompt_logits(p[:i + 1])
        top2 = lg.topk(2).values
        if float(top2[0] - top2[1]) > 1e-3:  # skip exact near-ties
            assert preds[i] == int(lg.argmax()), i


def test_prefix_tier_restores_across_engines(tiny, tmp_path):
    from rocket_b200.kv.prefix_store import PrefixTier
    cfg, t = tiny
    p = _prompts(cfg, 1, L=300, seed=5)[0]
    a = _engine(cfg, t, prefix=True)
    ta = PrefixTier(a, str(tmp_path))
    a.attach_prefix_tier(ta)
    ref = a.generate([p], max_new_tokens=8)[0]
    assert ta.saved >= 4
    b = _engine(cfg, t, prefix=True)
    tb = PrefixTier(b, str(tmp_path))
    b.attach_prefix_tier(tb)
    out = b.generate([p], max_new_tokens=8)[0]
    assert tb.restored >= 4 and b.kv.hits() >= 4
    assert out == ref
    del ta, tb
    # corrupt the first record: the third engine recomputes and still agrees
    segd = os.path.join(str(tmp_path), "segments")
    seg = os.path.join(segd, sorted(os.listdir(segd))[0])
    with open(seg, "r+b") as f:
        f.seek(1000)
        x = f.read(1)
        f.seek(1000)
        f.write(bytes([x[0] ^ 0x55]))
    c = _engine(cfg, t, prefix=True)
    tc = PrefixTier(c, str(tmp_path))
    c.attach_prefix_tier(tc)
    assert c.generate([p], max_new_tokens=8)[0] == ref
    assert tc.restored == 0 and tc.stats()["checksum_failures"] == 1


@pytest.mark.parametrize("name", ["tiny-moe", "tiny-hybrid", "tiny-dsa", "tiny-mla"])
def test_session_checkpoint_and_resume(name, tmp_path):
    from rocket_b200.engine.scheduler import Status
    from rocket_b200.kv.prefix_store import SessionStore
    cfg = load_fuel(name).model
    t = init_fuel_tensors(cfg, 0)
    p = _prompts(cfg, 1, L=70, seed=9)[0]
    ref = _engine(cfg, t, name, graphs=False).generate([p], max_new_tokens=20)[0]
    a = _engine(cfg, t, name, graphs=False)
    r = a.add_request(p, 20)
    while len(r.output) < 8:
        a.step()
    assert r.status == Status.DECODE
    if name == "tiny-moe":
        key = SessionStore(a, str(tmp_path)).save(r)
    else:
        # the transactional path (kv.state_txn): prepare / commit / index, authenticated restore
        from rocket_b200.kv.state_txn import DistributedTxn
        SessionStore(a, str(tmp_path)).save_txn(r, "sess0", DistributedTxn(str(tmp_path / "txn")))
    a.abort(r)
    b = _engine(cfg, t, name, graphs=False)
    if name == "tiny-moe":
        r2 = SessionStore(b, str(tmp_path)).resume(key)
    else:
        r2 = SessionStore(b, str(tmp_path)).resume_txn("sess0", DistributedTxn(str(tmp_path / "txn")))
    while b.sched.has_work():
        b.step()
    assert r2.output == ref, (r2.output, ref)


def test_engine_faults_latch_after_a_failed_step():
    """A step that raises leaves the engine faulted: later steps refuse to run (the device
    state may be mid-step); spans of the steps before are recorded with their outcome."""
    from rocket_b200.engine import EngineFaulted
    from rocket_b200.utils.tracing import Tracer
    cfg = load_fuel("tiny-moe").model
    t = init_fuel_tensors(cfg, 0)
    eng = _engine(cfg, t, "tiny-moe", graphs=False)
    eng.tracer = Tracer()
    eng.add_request(_prompts(cfg, 1, L=20, seed=1)[0], 8)
    eng.step()
    real = eng._run

    def broken(sched):
        raise RuntimeError("injected host failure")
    eng._run = broken
    with pytest.raises(RuntimeError, match="injected"):
        eng.step()
    eng._run = real
    assert eng.phase == "faulted"
    with pytest.raises(EngineFaulted):
        eng.step()
    outcomes = [s[1]["outcome"] for s in eng.tracer.spans if s[0] == "step"]
    assert outcomes == ["ok", "error"]


def test_http_server_serves_the_engine():
    """The OpenAI-style front-end over a real engine: completions equal engine.generate."""
    from fastapi.testclient import TestClient

    from rocket_b200.serve import EngineLoop, build_app
    cfg = load_fuel("tiny-moe").model
    t = init_fuel_tensors(cfg, 0)
    prompts = _prompts(cfg, 2, L=30, seed=21)
    ref = _engine(cfg, t, "tiny-moe").generate(prompts, max_new_tokens=6)
    eng = _engine(cfg, t, "tiny-moe")
    loop = EngineLoop(eng).start()
    try:
        c = TestClient(build_app(loop, "tiny-moe"))
        for p, o in zip(prompts, ref):
            r = c.post("/v1/completions", json={"prompt": p, "max_tokens": 6})
            assert r.status_code == 200, r.text
            assert r.json()["choices"][0]["token_ids"] == o
        assert "generated_tokens_total" in c.get("/metrics").text
    finally:
        loop.stop()


@pytest.mark.parametrize("name", ["tiny-moe", "tiny-hybrid"])
def test_checksum_taps_identical_across_runs(name):
    """Run-to-run determinism of KV pages, hidden rows and step outputs (spec on), step by step."""
    from rocket_b200.utils.checksums import ChecksumTap, first_divergence
    cfg = load_fuel(name).model
    t = init_fuel_tensors(cfg, 0)
    prompts = _prompts(cfg, 3, L=45, seed=2)
    streams = []
    for _ in range(2):
        e = EngineConfig(max_batch=4, batch_buckets=[4], prefill_chunk=32, max_seq_len=256, prefix_cache=False,
                         spec_tokens=3)
        eng = LLMEngine.from_fuel(name, e, tensors=t, kv_pages=64, cfg_override=cfg)
        eng.checksums = ChecksumTap(eng, ["kv", "hidden", "spec"])
        eng.generate(prompts, max_new_tokens=8)
        streams.append(eng.checksums.records)
    assert len(streams[0]) > 3
    assert first_divergence(*streams) is None
