"""Native NVFP4 codec and the offline fuel materializer (C++) against the Python codec."""
import os

import pytest
import torch

from rocket_b200.fuel import nvfp4 as nv

rt = pytest.importorskip("rocket_b200._rt")


def test_e4m3_encoder_matches_torch():
    # every e4m3 value, every midpoint between neighbours (ties), and random values
    vals = torch.arange(0, 127, dtype=torch.uint8).view(torch.float8_e4m3fn).float()
    mids = (vals[1:] + vals[:-1]) / 2
    rnd = torch.rand(20000) * 448
    tiny = torch.rand(2000) * 0.02
    x = torch.cat([vals, mids, rnd, tiny, torch.tensor([0.0, 447.9, 448.0])])
    ref = nv.e4m3_encode(x)
    got = torch.tensor([rt.e4m3_from_float(float(v)) for v in x], dtype=torch.uint8)
    assert torch.equal(got, ref), (x[got != ref][:5], got[got != ref][:5], ref[got != ref][:5])
    back = torch.tensor([rt.e4m3_to_float(int(b)) for b in range(127)])
    assert torch.equal(back, vals)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_quantize_matches_python_codec(dtype):
    g = torch.Generator().manual_seed(1)
    w = torch.randn(67, 256, generator=g) * 0.02
    w[3] = 0                       # an all-zero row (zero block scales)
    w[5, :16] *= 1e-4              # a block whose scale is an e4m3 subnormal
    w[7, 40] = 3.0                 # an outlier that sets the tensor scale
    w = w.to(dtype)
    pk, sf, gs = nv.quantize_nvfp4(w)
    name = {torch.float32: "F32", torch.bfloat16: "BF16", torch.float16: "F16"}[dtype]
    buf = w.contiguous().view(torch.uint8).numpy()
    pk2, sf2, gs2 = rt.quantize_nvfp4(buf, name, 67, 256, 0.0, 4)
    assert torch.tensor(gs2) == torch.tensor(gs, dtype=torch.float32)
    assert torch.equal(torch.from_numpy(sf2), sf)
    assert torch.equal(torch.from_numpy(pk2), pk)


def test_swizzle_matches_python():
    sf = torch.randint(0, 127, (300, 20), dtype=torch.uint8)
    assert torch.equal(torch.from_numpy(rt.swizzle_sf(sf.numpy())), nv.swizzle_sf(sf))


def test_materialize_fuel_roundtrip(tmp_path):
    from rocket_b200.config import load_fuel
    from rocket_b200.fuel.materialize import materialize, verify
    from rocket_b200.fuel.safetensors_io import load_dir, save_dir
    from rocket_b200.models import init_fuel_tensors
    cfg = load_fuel("tiny-moe").model
    t = init_fuel_tensors(cfg, 0)
    # an unquantized "upstream" checkpoint: every linear in bf16 (the fp32 masters, rounded)
    src = {}
    for k, v in t.items():
        if k.startswith("master."):
            continue
        base = k[:-len(".weight")] if k.endswith(".weight") else None
        if base and "master." + base in t:
            src[k] = t["master." + base].bfloat16()
        elif k.endswith((".weight_scale", ".weight_scale_2")):
            continue
        else:
            src[k] = v
    src["layers.0.attn_norm.weight"] = src["layers.0.attn_norm.weight"].float()  # an fp32 tensor: cast
    sdir, odir = str(tmp_path / "src"), str(tmp_path / "out")
    save_dir(src, sdir, shard_bytes=1 << 20)
    rep = materialize(sdir, odir, cfg.weight_format, shard_bytes=2 << 20, threads=3)
    assert rep["quantized"] > 0 and rep["max_rel_err"] < 0.2, rep
    out = load_dir(odir)
    assert out["layers.0.attn_norm.weight"].dtype == torch.bfloat16
    n_checked = 0
    for k in src:
        if not k.endswith(".weight"):
            continue
        base = k[:-len(".weight")]
        if base + ".weight_scale" in out:
            pk, sf, gs = nv.quantize_nvfp4(src[k])
            assert torch.equal(out[k], pk), k
            assert torch.equal(out[base + ".weight_scale"].view(torch.uint8), sf), k
            assert out[base + ".weight_scale_2"].item() == torch.tensor(gs, dtype=torch.float32).item()
            n_checked += 1
        else:
            assert torch.equal(out[k].float(), src[k].float()), k
    assert n_checked == rep["quantized"]
    assert verify(odir) == []
    # a flipped byte in a shard is caught
    shard = sorted(f for f in os.listdir(odir) if f.endswith(".safetensors"))[0]
    p = os.path.join(odir, shard)
    with open(p, "r+b") as f:
        f.seek(os.path.getsize(p) - 3)
        b = f.read(1)
        f.seek(-1, 1)
        f.write(bytes([b[0] ^ 0x10]))
    assert verify(odir) == [shard]


def test_materialize_refuses_bad_inputs(tmp_path):
    from rocket_b200.fuel.safetensors_io import save_file
    p = str(tmp_path / "a.safetensors")
    save_file({"x.weight": torch.zeros(4, 20)}, p)   # 20 columns: not a multiple of 16
    with pytest.raises(Exception):
        rt.materialize_nvfp4([p], str(tmp_path / "o"), {"x"})
    with pytest.raises(Exception):
        rt.materialize_nvfp4([p], str(tmp_path / "o"), {"missing"})


def test_quantize_fuel_cli(tmp_path):
    import json
    import subprocess
    import sys
    from rocket_b200.fuel.safetensors_io import load_dir, save_file
    src = str(tmp_path / "in.safetensors")
    save_file({"layers.0.mlp.gate_proj.weight": torch.randn(32, 64) * 0.02,
               "layers.0.attn_norm.weight": torch.ones(64)}, src)
    out = str(tmp_path / "fuel")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-m", "rocket_b200", "quantize-fuel", "--src", src, "--out", out,
                        "--fuel", "glm-moe-small"], capture_output=True, text=True, cwd=root, timeout=300)
    assert r.returncode == 0, r.stderr
    rep = json.loads(r.stdout.strip().splitlines()[-1])
    assert rep["quantized"] == 1
    t = load_dir(out)
    assert t["layers.0.mlp.gate_proj.weight"].shape == (32, 32)
    r = subprocess.run([sys.executable, "-m", "rocket_b200", "verify-fuel", "--dir", out], capture_output=True,
                       text=True, cwd=root, timeout=300)
    assert r.returncode == 0 and json.loads(r.stdout)["bad_shards"] == []


def test_materialize_fp8_rows_matches_python(tmp_path):
    from rocket_b200.fuel.materialize import materialize
    from rocket_b200.fuel.safetensors_io import load_dir, save_file
    from rocket_b200.models.weights import quantize_fp8_rows
    g = torch.Generator().manual_seed(3)
    w = torch.randn(96, 80, generator=g) * 0.05
    w[4] = 0
    src = str(tmp_path / "in.safetensors")
    save_file({"layers.0.attn.q_proj.weight": w.bfloat16(), "layers.0.mlp.gate_proj.weight": w[:, :64].clone()}, src)
    rep = materialize(src, str(tmp_path / "out"), {"attention": "fp8", "dense": "nvfp4"})
    assert rep["quantized"] == 2
    out = load_dir(str(tmp_path / "out"))
    q, s = quantize_fp8_rows(w.bfloat16())
    assert out["layers.0.attn.q_proj.weight"].dtype == torch.float8_e4m3fn
    assert torch.equal(out["layers.0.attn.q_proj.weight"].view(torch.uint8), q.view(torch.uint8))
    assert torch.equal(out["layers.0.attn.q_proj.weight_scale"], s)
    assert "layers.0.mlp.gate_proj.weight_scale_2" in out
