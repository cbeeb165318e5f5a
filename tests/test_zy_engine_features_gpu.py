"""Engine features on the GPU: agent-trace replay over the prefix cache, the sentinel
check, the generate CLI, streamed experts, teacher-forced NLL, request fork and
detach / attach, attention biases, programmatic dependent launch, host-only
speculation on models without an MTP head, the draft-model source and the adaptive
draft chain.  Kept in one module that runs after the kernel / engine / speculation
suites."""
import pytest
import torch

from rocket_b200 import ops
from rocket_b200.config import EngineConfig, load_fuel
from rocket_b200.engine import LLMEngine
from rocket_b200.models import ReferenceModel, init_fuel_tensors

pytestmark = pytest.mark.gpu

K = 3


@pytest.fixture(scope="module")
def tiny():
    cfg = load_fuel("tiny-moe").model
    return cfg, init_fuel_tensors(cfg, 0)


def _engine(cfg, t, name="tiny-moe", **kw):
    """Engine over fuel tensors `t` (max_batch 4 or kw, graphs on unless graphs=False)."""
    e = EngineConfig(max_batch=kw.get("max_batch", 8), batch_buckets=kw.get("buckets", [1, 2, 4, 8]),
                     prefill_chunk=kw.get("chunk", 512), max_seq_len=kw.get("max_seq_len", 256),
                     cuda_graphs=kw.get("graphs", True), prefix_cache=kw.get("prefix", False),
                     spec_tokens=kw.get("spec", 0))
    return LLMEngine.from_fuel(name, e, tensors=t, kv_pages=kw.get("pages", 64), cfg_override=cfg)


def _prompts(cfg, n=4, L=64, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, cfg.vocab_size, (L,), generator=g).tolist() for _ in range(n)]


def test_agent_trace_replay_hits_the_prefix_cache(tiny):
    """A forked-prefix agent trace through the engine: every request completes with the
    trace's token counts and the shared root prefix comes from the prefix cache."""
    from rocket_b200.engine.agent_workload import EngineBackend, agent_trace, replay_trace
    cfg, t = tiny
    eng = _engine(cfg, t, prefix=True, pages=128, max_batch=4, buckets=[4], max_seq_len=320)
    ev = agent_trace(concurrency=4, depth=2, prefix_tokens=128, duration_steps=12, seed=0, max_context=300)
    res = replay_trace(EngineBackend(eng), ev, cfg.vocab_size)
    ops.check_errors()
    assert res["output_tokens"] == sum(e["n_tokens"] for e in ev if e["event"] == "decode")
    assert res["prompt_cache_fraction"] > 0.3, res
    eng.release_graphs()


def test_sentinel_check_passes_on_a_correct_model(tiny, monkeypatch):
    """ROCKET_SENTINEL=1: expert GEMM outputs are NaN-filled before every MoE layer and
    every routed row must have been written (eager steps)."""
    monkeypatch.setenv("ROCKET_SENTINEL", "1")
    cfg, t = tiny
    eng = _engine(cfg, t)
    assert eng.model.sentinel and not eng.use_graphs
    g = torch.Generator().manual_seed(4)
    prompts = [torch.randint(0, cfg.vocab_size, (40,), generator=g).tolist() for _ in range(3)]
    out = eng.generate(prompts, max_new_tokens=6)
    monkeypatch.setenv("ROCKET_SENTINEL", "0")
    assert out == _engine(cfg, t).generate(prompts, max_new_tokens=6)


def test_generate_cli_batch_and_prefix_tier(tmp_path):
    """The decode CLI over a JSON-lines prompt list, replicated by --batch, with the
    persistent prefix tier attached: one output per request, equal for equal prompts."""
    import json
    import subprocess
    import sys
    pl = tmp_path / "prompts.jsonl"
    pl.write_text("\n".join(json.dumps(list(range(1 + i, 70 + i))) for i in range(2)) + "\n")
    cmd = [sys.executable, "-m", "rocket_b200", "generate", "--fuel", "tiny-moe", "--prompt-list", str(pl),
           "--batch", "2", "--max-new-tokens", "5", "--prefix-cache-dir", str(tmp_path / "tier"),
           "--result-json", str(tmp_path / "r.json")]
    out = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    res = json.loads((tmp_path / "r.json").read_text())
    assert res["requests"] == 4 and [len(o) for o in res["outputs"]] == [5] * 4
    assert res["outputs"][0] == res["outputs"][1] and res["outputs"][2] == res["outputs"][3]


def _streamed(cfg, t, slots, **kw):
    e = EngineConfig(max_batch=kw.get("max_batch", 8), prefill_chunk=kw.get("chunk", 512), max_seq_len=256,
                     prefix_cache=False, expert_cache_slots=slots)
    return LLMEngine.from_fuel("tiny-moe", e, tensors=t, kv_pages=64, cfg_override=cfg)


def test_streamed_experts_equal_resident_with_room_for_a_step(tiny):
    """Slots for every expert: one pass per layer, results bit-identical to the resident
    model (the slot permutation changes no row's arithmetic)."""
    cfg, t = tiny
    ref = _engine(cfg, t, graphs=False)
    eng = _streamed(cfg, t, cfg.num_experts)
    assert not eng.use_graphs and eng.model.streamer is not None
    for p in _prompts(cfg, 2, seed=5):
        assert torch.equal(eng.prompt_logits(p), ref.prompt_logits(p))
    prompts = _prompts(cfg, 4, 48, seed=6)
    assert eng.generate(prompts, max_new_tokens=12) == ref.generate(prompts, max_new_tokens=12)
    st = eng.model.streamer.stats()
    assert st["hits"] > 0 and st["passes"] >= st["layers"]


def test_streamed_experts_with_few_slots_track_resident(tiny):
    """Two slots per layer: several passes per layer and LRU evictions; the residual picks
    up one extra bf16 rounding per pass, so logits stay close to the resident model."""
    cfg, t = tiny
    ref = _engine(cfg, t, graphs=False)
    eng = _streamed(cfg, t, 2)
    for p in _prompts(cfg, 2, seed=7):
        a, b = eng.prompt_logits(p), ref.prompt_logits(p)
        # an extra bf16 rounding of the residual per pass can flip a few NVFP4 codes downstream
        assert torch.nn.functional.cosine_similarity(a, b, 0).item() > 0.99
    st = eng.model.streamer.stats()
    assert st["evictions"] > 0 and st["passes"] > st["layers"]
    assert eng.model.weight_bytes() < ref.model.weight_bytes()


def test_teacher_nll_matches_prompt_logits(tiny):
    """teacher_nll over chunked prefill equals -log softmax of the prefix logits, and a
    model scores its own greedy continuation below a random one."""
    cfg, t = tiny
    eng = _engine(cfg, t, graphs=False)  # teacher_nll chunks by the sampled-row limit (max_batch rows)
    p = _prompts(cfg, 1, 90, seed=8)[0]
    nll = eng.teacher_nll(p)
    assert len(nll) == len(p) - 1
    for i in (5, 39, 40, 88):
        lg = eng.prompt_logits(p[:i + 1])
        ref = -torch.log_softmax(lg.double(), 0)[p[i + 1]].item()
        # chunked vs one-shot prefill: attention work splits differ, so NVFP4 codes may flip
        assert abs(nll[i] - ref) < 0.05 + 0.01 * abs(ref), (i, nll[i], ref)
    cont = eng.generate([p[:40]], max_new_tokens=24)[0]
    own = sum(eng.teacher_nll(p[:40] + cont)[39:]) / 24
    rnd = sum(nll[39:63]) / 24
    assert own < rnd


def test_fork_continues_like_its_parent(tiny):
    """A fork taken mid-generation (boundary page copied, full pages shared) decodes the
    same greedy continuation as its parent and as an unforked run."""
    cfg, t = tiny
    p = _prompts(cfg, 1, 45, seed=9)[0]
    ref = _engine(cfg, t).generate([p], max_new_tokens=20)[0]
    eng = _engine(cfg, t)
    r = eng.add_request(p, 20)
    while len(r.output) < 6:
        eng.step()
    c = eng.fork(r, 20 - len(r.output))
    while eng.sched.has_work():
        eng.step()
    assert r.output == ref and c.output == ref


def test_attention_bias_tracks_oracle():
    """q/k/v biases (GLM-4.5's attention_bias) are added to this rank's QKV output rows."""
    from rocket_b200.config.schema import model_config
    cfg = model_config("tiny-moe", attention_bias=True)
    t = init_fuel_tensors(cfg, 0)
    e = EngineConfig(max_batch=8, prefill_chunk=512, max_seq_len=256, prefix_cache=False)
    eng = LLMEngine.from_fuel("tiny-moe", e, tensors=t, kv_pages=64, cfg_override=cfg)
    assert eng.model.layers[0].qkv_bias is not None
    emu = ReferenceModel(cfg, t, quantized=True, emulate_gpu=True)
    for p in _prompts(cfg, 2, seed=10):
        got = eng.prompt_logits(p)
        ref = emu.logits(torch.tensor(p))[-1]
        cos = torch.nn.functional.cosine_similarity(got, ref, 0).item()
        rel = ((got - ref).norm() / ref.norm()).item()
        assert cos > 0.97 and rel < 0.3, (cos, rel)
    rnd = LLMEngine.from_fuel("tiny-moe", e, kv_pages=64, cfg_override=cfg)  # random-init path
    assert len(rnd.generate(_prompts(cfg, 1, seed=11), max_new_tokens=4)[0]) == 4


@pytest.mark.parametrize("graphs", [True, False])
def test_programmatic_dependent_launch_keeps_results(tiny, graphs):
    """With PDL on, each hot kernel may be scheduled while its predecessor drains and
    waits for it on the device: the tokens are those of serialized launches."""
    if not ops.pdl_supported():
        pytest.skip("built without -DRKT_PDL (the kernels carry no device-side waits)")
    cfg, t = tiny
    prompts = _prompts(cfg, 4, 48, seed=14)
    ref = _engine(cfg, t, graphs=graphs).generate(prompts, max_new_tokens=12)
    ops.set_pdl(True)
    try:
        assert ops.pdl_enabled()
        got = _engine(cfg, t, graphs=graphs).generate(prompts, max_new_tokens=12)
        ops.check_errors()
    finally:
        ops.set_pdl(False)
    assert got == ref


@pytest.mark.parametrize("name", ["tiny-moe", "tiny-hybrid"])
def test_detached_request_resumes_exactly(name):
    """A request parked mid-generation (KV pages kept, DeltaNet state in host memory)
    while another request runs resumes to the same greedy output as an uninterrupted run."""
    cfg = load_fuel(name).model
    t = init_fuel_tensors(cfg, 0)
    e = EngineConfig(max_batch=4, prefill_chunk=512, max_seq_len=256, prefix_cache=False, batch_buckets=[1, 2, 4])
    p, other = _prompts(cfg, 2, 40, seed=15)
    ref = LLMEngine.from_fuel(name, e, tensors=t, kv_pages=64, cfg_override=cfg).generate([p], max_new_tokens=16)[0]
    eng = LLMEngine.from_fuel(name, e, tensors=t, kv_pages=64, cfg_override=cfg)
    r = eng.add_request(p, 16)
    while len(r.output) < 5:
        eng.step()
    d = eng.detach(r)
    eng.generate([other], max_new_tokens=8)       # reuses the freed slot meanwhile
    eng.attach(d)
    while eng.sched.has_work():
        eng.step()
    assert r.output == ref


@pytest.mark.parametrize("name", ["tiny-moe", "tiny-hybrid"])
@pytest.mark.parametrize("source", ["file", "prompt_lookup"])
def test_host_drafted_speculation_without_an_mtp_head(name, source):
    """A model without an MTP head verifies host drafts (a reference generation, or
    prompt lookup on prompts that repeat a block): verify + accept + KV rollback
    (+ DeltaNet commit) run, the MTP passes do not, and the output stays greedy."""
    from rocket_b200.config.schema import model_config
    from rocket_b200.engine.drafts import DraftFile
    cfg = model_config(name, mtp_layers=0)
    t = init_fuel_tensors(cfg, 0)
    g = torch.Generator().manual_seed(12)
    block = torch.randint(0, cfg.vocab_size, (12,), generator=g).tolist()
    prompts = [torch.randint(0, cfg.vocab_size, (8,), generator=g).tolist() + block * 3 for _ in range(4)]
    ref = _engine(cfg, t, name, max_batch=4, buckets=[4]).generate(prompts, max_new_tokens=24)
    e = EngineConfig(max_batch=4, batch_buckets=[4], prefill_chunk=512, max_seq_len=256, prefix_cache=False,
                     spec_tokens=K, draft_source="prompt_lookup")
    eng = LLMEngine.from_fuel(name, e, tensors=t, kv_pages=64, cfg_override=cfg)
    assert eng.model.mtp is None and not eng.model.has_mtp
    if source == "file":
        eng.set_draft_source(DraftFile({DraftFile.prompt_key(p): o for p, o in zip(prompts, ref)}))
    reqs = [eng.add_request(p, 24) for p in prompts]
    while eng.sched.has_work():
        eng.step()
    ops.check_errors()
    sm = eng.spec_summary(reqs)
    same = sum(int(a == b) for r, rr in zip(reqs, ref) for a, b in zip(r.output, rr)) / sum(len(o) for o in ref)
    assert same > 0.9, (same, sm)
    if source == "file":
        assert sm["acceptance"] > 0.8, sm
    eng.release_graphs()
    with pytest.raises(ValueError):
        LLMEngine.from_fuel(name, EngineConfig(max_batch=4, batch_buckets=[4], max_seq_len=256, prefix_cache=False,
                                               spec_tokens=K), tensors=t, kv_pages=64, cfg_override=cfg)


def test_draft_model_source():
    """A separate draft model (here the target's own weights, so its greedy drafts are
    the target's continuation) drafts for all decoding sequences in one batched run per
    step; nearly every draft is accepted and the output stays greedy."""
    from rocket_b200.config.schema import model_config
    from rocket_b200.engine.drafts import DraftModel
    cfg = model_config("tiny-moe", mtp_layers=0)
    t = init_fuel_tensors(cfg, 0)
    prompts = _prompts(cfg, 4, 40, seed=13)
    ref = _engine(cfg, t, "tiny-moe", max_batch=4, buckets=[4]).generate(prompts, max_new_tokens=20)
    draft = LLMEngine.from_fuel("tiny-moe", EngineConfig(max_batch=4, batch_buckets=[4], prefill_chunk=512,
                                                         max_seq_len=256, prefix_cache=True),
                                tensors=t, kv_pages=96, cfg_override=cfg)
    e = EngineConfig(max_batch=4, batch_buckets=[4], prefill_chunk=512, max_seq_len=256, prefix_cache=False,
                     spec_tokens=K, draft_source="history")
    eng = LLMEngine.from_fuel("tiny-moe", e, tensors=t, kv_pages=64, cfg_override=cfg)
    src = DraftModel(draft)
    eng.set_draft_source(src)
    reqs = [eng.add_request(p, 20) for p in prompts]
    while eng.sched.has_work():
        eng.step()
    ops.check_errors()
    sm = eng.spec_summary(reqs)
    same = sum(int(a == b) for r, rr in zip(reqs, ref) for a, b in zip(r.output, rr)) / sum(len(o) for o in ref)
    assert same > 0.9, (same, sm)
    assert sm["acceptance"] > 0.7 and src.steps > 0, sm
    eng.release_graphs()
    draft.release_graphs()



def test_adaptive_draft_chain_keeps_greedy_output():
    """The adaptive chain (prompt lookup demoted when it keeps failing, then history,
    then the MTP drafts) verifies on the device; the output stays greedy."""
    cfg = load_fuel("tiny-moe").model
    t = init_fuel_tensors(cfg, 0)
    g = torch.Generator().manual_seed(11)
    block = torch.randint(0, cfg.vocab_size, (12,), generator=g).tolist()
    prompts = [torch.randint(0, cfg.vocab_size, (8,), generator=g).tolist() + block * 3 for _ in range(4)]
    ref = _engine(cfg, t, max_batch=4, buckets=[4]).generate(prompts, max_new_tokens=24)
    eng = _engine(cfg, t, max_batch=4, buckets=[4], spec=K)
    eng.set_draft_source("adaptive:prompt_lookup+history+mtp")
    reqs = [eng.add_request(p, 24) for p in prompts]
    while eng.sched.has_work():
        eng.step()
    ops.check_errors()
    same = sum(int(a == b) for r, rr in zip(reqs, ref) for a, b in zip(r.output, rr)) / sum(len(o) for o in ref)
    assert same > 0.9, (same, eng.spec_summary(reqs))
